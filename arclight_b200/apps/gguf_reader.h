// Minimal GGUF reader for the Qwen3 Q4_0 models of the engine (header only).
//
// The reference reads a model in llm_model::load_model / load_all_tensors
// (src/model.cpp:130-335: magic, u32 version, u64 tensor and key/value counts,
// the key/values, the tensor infos; the data section starts at the first
// multiple of the alignment -- general.alignment, default 32 -- after the
// infos, and each tensor's offset is relative to it).  Keys and tensor names are
// those of models/qwen3.cpp:7-45.  This reader keeps the scalar key/values
// (strings and arrays are skipped) and maps the file once (mmap); the engine
// takes the weights through alb_engine_set_weight_blocks / _set_norm_weights.
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

namespace gguf {

enum : uint32_t { T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STRING, T_ARRAY, T_U64, T_I64, T_F64 };
enum : uint32_t { GGML_F32 = 0, GGML_F16 = 1, GGML_Q4_0 = 2 };

struct Tensor {
    std::vector<uint64_t> ne;   // ne[0] innermost
    uint32_t type = 0;
    uint64_t offset = 0;        // absolute file offset
    uint64_t nbytes = 0;
};

class File {
  public:
    explicit File(const std::string & path) {
        fd_ = open(path.c_str(), O_RDONLY);
        if (fd_ < 0) throw std::runtime_error("cannot open " + path);
        struct stat st;
        if (fstat(fd_, &st) != 0) throw std::runtime_error("cannot stat " + path);
        size_ = (size_t)st.st_size;
        base_ = static_cast<const uint8_t *>(mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0));
        if (base_ == MAP_FAILED) throw std::runtime_error("cannot map " + path);
        parse();
    }
    ~File() {
        if (base_ && base_ != MAP_FAILED) munmap(const_cast<uint8_t *>(base_), size_);
        if (fd_ >= 0) close(fd_);
    }
    File(const File &) = delete;
    File & operator=(const File &) = delete;

    bool has_key(const std::string & k) const { return num_.count(k) != 0; }
    double num(const std::string & k) const {
        auto it = num_.find(k);
        if (it == num_.end()) throw std::runtime_error("missing key " + k);
        return it->second;
    }
    double num_or(const std::string & k, double d) const { return has_key(k) ? num_.at(k) : d; }
    const std::string & str(const std::string & k) const {
        static const std::string empty;
        auto it = str_.find(k);
        return it == str_.end() ? empty : it->second;
    }
    bool has_tensor(const std::string & n) const { return tensors_.count(n) != 0; }
    const Tensor & tensor(const std::string & n) const {
        auto it = tensors_.find(n);
        if (it == tensors_.end()) throw std::runtime_error("missing tensor " + n);
        return it->second;
    }
    const uint8_t * data(const Tensor & t) const { return base_ + t.offset; }

  private:
    int fd_ = -1;
    size_t size_ = 0, pos_ = 0;
    const uint8_t * base_ = nullptr;
    std::map<std::string, double> num_;
    std::map<std::string, std::string> str_;
    std::map<std::string, Tensor> tensors_;

    void need(size_t n) const {
        if (pos_ + n > size_) throw std::runtime_error("truncated GGUF file");
    }
    template <typename T> T rd() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, base_ + pos_, sizeof(T));
        pos_ += sizeof(T);
        return v;
    }
    std::string rd_str() {
        const uint64_t n = rd<uint64_t>();
        need(n);
        std::string s(reinterpret_cast<const char *>(base_ + pos_), n);
        pos_ += n;
        return s;
    }
    static size_t scalar_size(uint32_t t) {
        switch (t) {
            case T_U8: case T_I8: case T_BOOL: return 1;
            case T_U16: case T_I16: return 2;
            case T_U32: case T_I32: case T_F32: return 4;
            case T_U64: case T_I64: case T_F64: return 8;
            default: return 0;
        }
    }
    double rd_num(uint32_t t) {
        switch (t) {
            case T_U8: return rd<uint8_t>();
            case T_I8: return rd<int8_t>();
            case T_BOOL: return rd<uint8_t>();
            case T_U16: return rd<uint16_t>();
            case T_I16: return rd<int16_t>();
            case T_U32: return rd<uint32_t>();
            case T_I32: return rd<int32_t>();
            case T_F32: return rd<float>();
            case T_U64: return (double)rd<uint64_t>();
            case T_I64: return (double)rd<int64_t>();
            case T_F64: return rd<double>();
            default: throw std::runtime_error("unknown GGUF value type");
        }
    }
    void skip_value(uint32_t t) {
        if (t == T_STRING) { rd_str(); return; }
        if (t == T_ARRAY) {
            const uint32_t et = rd<uint32_t>();
            const uint64_t n = rd<uint64_t>();
            if (et == T_STRING) { for (uint64_t i = 0; i < n; ++i) rd_str(); return; }
            const size_t s = scalar_size(et);
            if (!s) throw std::runtime_error("unsupported GGUF array element type");
            need(s * n);
            pos_ += s * n;
            return;
        }
        rd_num(t);
    }
    void parse() {
        need(4);
        if (std::memcmp(base_, "GGUF", 4) != 0) throw std::runtime_error("not a GGUF file");
        pos_ = 4;
        const uint32_t version = rd<uint32_t>();
        if (version != 2 && version != 3) throw std::runtime_error("unsupported GGUF version");
        const uint64_t n_tensors = rd<uint64_t>(), n_kv = rd<uint64_t>();
        for (uint64_t i = 0; i < n_kv; ++i) {
            const std::string key = rd_str();
            const uint32_t t = rd<uint32_t>();
            if (t == T_STRING) str_[key] = rd_str();
            else if (t == T_ARRAY) skip_value(t);
            else num_[key] = rd_num(t);
        }
        const uint64_t align = (uint64_t)num_or("general.alignment", 32);
        if (align == 0 || (align & (align - 1))) throw std::runtime_error("bad GGUF alignment");
        std::vector<std::pair<std::string, Tensor>> infos;
        for (uint64_t i = 0; i < n_tensors; ++i) {
            Tensor t;
            const std::string name = rd_str();
            const uint32_t nd = rd<uint32_t>();
            for (uint32_t d = 0; d < nd; ++d) t.ne.push_back(rd<uint64_t>());
            t.type = rd<uint32_t>();
            t.offset = rd<uint64_t>();
            infos.emplace_back(name, t);
        }
        const uint64_t data0 = (pos_ + align - 1) / align * align;
        for (auto & [name, t] : infos) {
            uint64_t count = 1;
            for (uint64_t x : t.ne) count *= x;
            if (t.type == GGML_F32) t.nbytes = count * 4;
            else if (t.type == GGML_F16) t.nbytes = count * 2;
            else if (t.type == GGML_Q4_0) {
                if (t.ne.empty() || t.ne[0] % 32) throw std::runtime_error("bad Q4_0 row length in " + name);
                t.nbytes = count / 32 * 18;
            } else {
                throw std::runtime_error("unsupported tensor type in " + name);
            }
            t.offset += data0;
            if (t.offset + t.nbytes > size_) throw std::runtime_error("tensor " + name + " runs past the end");
            tensors_[name] = t;
        }
    }
};

}  // namespace gguf
