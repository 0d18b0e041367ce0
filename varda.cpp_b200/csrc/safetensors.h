// Read-only safetensors container with strict consumption tracking: the model-file format of
// varda.cpp (reference src/varda/format.h:15-73). The file is mmap'd; tensors are views into the
// mapping. Loading is strict: every tensor must be take()n or the load fails.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <set>
#include <string>
#include <vector>

namespace vb {

enum class DType { F32, F16, BF16, F64, I64, I32, I16, I8, U8, BOOL };
const char* dtype_name(DType t);
size_t dtype_size(DType t);

struct TensorView {
    std::string name;
    DType dtype = DType::F32;
    std::vector<int64_t> shape;
    const void* data = nullptr;  // into the mapping
    size_t nbytes = 0;
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t s : shape) n *= s;
        return n;
    }
    std::string shape_str() const;
    template <class T> const T* as() const { return static_cast<const T*>(data); }
};

class SafeTensorsFile {
public:
    explicit SafeTensorsFile(const std::string& path);
    ~SafeTensorsFile();
    SafeTensorsFile(const SafeTensorsFile&) = delete;
    SafeTensorsFile& operator=(const SafeTensorsFile&) = delete;

    const std::string& path() const { return path_; }
    const std::map<std::string, std::string>& metadata() const { return meta_; }
    std::string metadata(const std::string& key) const;  // throws when missing
    bool has(const std::string& name) const { return tensors_.count(name) != 0; }
    const TensorView& peek(const std::string& name) const;
    const TensorView& take(const std::string& name);
    const TensorView& take(const std::string& name, DType dtype, const std::vector<int64_t>& shape);
    std::vector<std::string> names() const;
    std::vector<std::string> unconsumed() const;
    void require_all_consumed() const;
    // Populates the page tables of the whole mapping with `threads` parallel readers (0: 16;
    // VB_PREFETCH_THREADS overrides, 0 there disables), so later reads fault on nothing.
    void prefetch(int threads = 0) const;

private:
    std::string path_;
    int fd_ = -1;
    void* map_ = nullptr;
    size_t size_ = 0;
    std::map<std::string, std::string> meta_;
    std::map<std::string, TensorView> tensors_;
    std::set<std::string> consumed_;
};

}  // namespace vb
