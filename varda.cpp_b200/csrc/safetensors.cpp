// safetensors reader (the container format of varda.cpp's converted model files; the layout is the
// published safetensors specification: an 8-byte little-endian header length N, N bytes of JSON
// {name: {dtype, shape, data_offsets: [begin, end)}, "__metadata__": {str: str}}, then the data
// section, offsets relative to its start).
//
// The file is mapped read-only and tensors are views of the mapping. Every header entry is checked
// before any tensor is handed out: a known dtype, non-negative dimensions whose product does not
// overflow, offsets inside the data section whose span equals the element count times the element
// size, natural alignment of the data, and no two tensors sharing bytes. Consumption is tracked by
// name, so a loader can insist that every tensor of the file was used.
#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "common.h"
#include "json.h"

namespace vb {

namespace {

// dtype names of the specification and their element sizes
DType dtype_from(const std::string& s, bool& ok) {
    ok = true;
    if (s == "F32") return DType::F32;
    if (s == "F16") return DType::F16;
    if (s == "BF16") return DType::BF16;
    if (s == "F64") return DType::F64;
    if (s == "I64") return DType::I64;
    if (s == "I32") return DType::I32;
    if (s == "I16") return DType::I16;
    if (s == "I8") return DType::I8;
    if (s == "U8") return DType::U8;
    if (s == "BOOL") return DType::BOOL;
    ok = false;
    return DType::F32;
}

}  // namespace

const char* dtype_name(DType t) {
    switch (t) {
        case DType::F32: return "F32";
        case DType::F16: return "F16";
        case DType::BF16: return "BF16";
        case DType::F64: return "F64";
        case DType::I64: return "I64";
        case DType::I32: return "I32";
        case DType::I16: return "I16";
        case DType::I8: return "I8";
        case DType::U8: return "U8";
        case DType::BOOL: return "BOOL";
    }
    return "?";
}
size_t dtype_size(DType t) {
    switch (t) {
        case DType::F64:
        case DType::I64: return 8;
        case DType::F32:
        case DType::I32: return 4;
        case DType::F16:
        case DType::BF16:
        case DType::I16: return 2;
        case DType::I8:
        case DType::U8:
        case DType::BOOL: return 1;
    }
    return 0;
}

std::string TensorView::shape_str() const {
    std::string s;
    for (int64_t d : shape) s += (s.empty() ? "" : ", ") + std::to_string(d);
    return "[" + s + "]";
}

SafeTensorsFile::SafeTensorsFile(const std::string& path) : path_(path) {
    auto invalid = [&](const std::string& why) { fail(kFormat, "safetensors file " + path + ": " + why); };
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) fail(kFormat, "cannot open " + path + " (" + std::strerror(errno) + ")");
    try {
        struct stat st {};
        if (::fstat(fd_, &st) != 0) invalid("cannot stat");
        size_ = size_t(st.st_size);
        if (size_ < 8) invalid("shorter than the 8-byte header length");
        map_ = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (map_ == MAP_FAILED) {
            map_ = nullptr;
            invalid(std::string("cannot map (") + std::strerror(errno) + ")");
        }
        const unsigned char* bytes = static_cast<const unsigned char*>(map_);
        uint64_t hlen = 0;
        for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | bytes[i];  // little-endian on any host
        if (hlen > size_ - 8) invalid("header of " + std::to_string(hlen) + " bytes runs past the end of the file");
        const char* h = reinterpret_cast<const char*>(bytes + 8);
        const json::Value header = json::parse(h, h + hlen);
        if (header.kind != json::Value::Object) invalid("the header is not a JSON object");
        const size_t data_begin = 8 + size_t(hlen), data_len = size_ - data_begin;

        std::vector<std::pair<uint64_t, uint64_t>> spans;  // for the overlap check
        for (const auto& [name, e] : header.obj) {
            if (name == "__metadata__") {
                if (e.kind != json::Value::Object) invalid("__metadata__ is not an object");
                for (const auto& [k, v] : e.obj) meta_[k] = v.as_str("__metadata__ value");
                continue;
            }
            const std::string what = "tensor '" + name + "'";
            if (e.kind != json::Value::Object) invalid(what + ": entry is not an object");
            TensorView t;
            t.name = name;
            bool ok = false;
            t.dtype = dtype_from(e.at("dtype").as_str("dtype"), ok);
            if (!ok) invalid(what + ": dtype '" + e.at("dtype").str + "' is not supported");
            t.shape = e.at("shape").int64_list("shape");
            uint64_t count = 1;
            for (int64_t d : t.shape) {
                if (d < 0) invalid(what + ": a dimension is negative");
                if (__builtin_mul_overflow(count, uint64_t(d), &count)) invalid(what + ": element count overflows");
            }
            uint64_t span = 0;
            if (__builtin_mul_overflow(count, uint64_t(dtype_size(t.dtype)), &span))
                invalid(what + ": byte size overflows");
            const std::vector<int64_t> off = e.at("data_offsets").int64_list("data_offsets");
            if (off.size() != 2 || off[0] < 0 || off[1] < off[0]) invalid(what + ": data_offsets must be [begin, end]");
            if (uint64_t(off[1]) > data_len) invalid(what + ": data ends past the data section");
            if (uint64_t(off[1] - off[0]) != span)
                invalid(what + ": " + std::to_string(off[1] - off[0]) + " bytes for " + t.shape_str() + " " +
                        dtype_name(t.dtype));
            t.nbytes = size_t(span);
            t.data = bytes + data_begin + size_t(off[0]);
            if (reinterpret_cast<uintptr_t>(t.data) % dtype_size(t.dtype)) invalid(what + ": data not naturally aligned");
            if (span) spans.emplace_back(uint64_t(off[0]), uint64_t(off[1]));
            tensors_.emplace(name, std::move(t));
        }
        std::sort(spans.begin(), spans.end());
        for (size_t i = 1; i < spans.size(); ++i)
            if (spans[i].first < spans[i - 1].second) invalid("two tensors share bytes of the data section");
    } catch (...) {
        if (map_) ::munmap(map_, size_);
        ::close(fd_);
        map_ = nullptr, fd_ = -1;
        throw;
    }
}

SafeTensorsFile::~SafeTensorsFile() {
    if (map_) ::munmap(map_, size_);
    if (fd_ >= 0) ::close(fd_);
}

std::string SafeTensorsFile::metadata(const std::string& key) const {
    const auto it = meta_.find(key);
    if (it == meta_.end()) fail(kFormat, path_ + ": the header's __metadata__ has no '" + key + "'");
    return it->second;
}

const TensorView& SafeTensorsFile::peek(const std::string& name) const {
    const auto it = tensors_.find(name);
    if (it == tensors_.end()) fail(kFormat, path_ + ": the model has no tensor '" + name + "'");
    return it->second;
}

const TensorView& SafeTensorsFile::take(const std::string& name) {
    const TensorView& t = peek(name);
    consumed_.insert(name);
    return t;
}

const TensorView& SafeTensorsFile::take(const std::string& name, DType dtype, const std::vector<int64_t>& shape) {
    const TensorView& t = take(name);
    if (t.dtype != dtype || t.shape != shape) {
        TensorView want;
        want.shape = shape;
        fail(kFormat, path_ + ": tensor '" + name + "' is " + dtype_name(t.dtype) + " " + t.shape_str() +
                          ", the model needs " + dtype_name(dtype) + " " + want.shape_str());
    }
    return t;
}

std::vector<std::string> SafeTensorsFile::names() const {
    std::vector<std::string> out;
    out.reserve(tensors_.size());
    for (const auto& kv : tensors_) out.push_back(kv.first);
    return out;
}

std::vector<std::string> SafeTensorsFile::unconsumed() const {
    std::vector<std::string> out;
    for (const auto& kv : tensors_)
        if (consumed_.find(kv.first) == consumed_.end()) out.push_back(kv.first);
    return out;
}

void SafeTensorsFile::require_all_consumed() const {
    const std::vector<std::string> left = unconsumed();
    if (left.empty()) return;
    std::string list;
    for (size_t i = 0; i < left.size() && i < 20; ++i) list += (i ? ", " : "") + left[i];
    if (left.size() > 20) list += ", ...";
    fail(kFormat, path_ + ": the engine used every tensor it needs but the file has " + std::to_string(left.size()) +
                      " more: " + list);
}

// The mapping is split into `threads` equal contiguous ranges; each thread asks the kernel to populate
// its range's page tables in one call (MADV_POPULATE_READ, Linux 5.14+) and otherwise reads one byte
// per page of it.
void SafeTensorsFile::prefetch(int threads) const {
    if (const char* e = std::getenv("VB_PREFETCH_THREADS"); e && *e) threads = std::atoi(e);
    else if (threads <= 0) threads = 16;
    if (threads <= 0 || !map_ || size_ == 0) return;
    const size_t page = size_t(::sysconf(_SC_PAGESIZE));
    const size_t pages = (size_ + page - 1) / page;
    const size_t n = std::min<size_t>(size_t(threads), pages);
    auto populate = [&](size_t i) {
        const size_t p0 = pages * i / n, p1 = pages * (i + 1) / n;
        char* lo = static_cast<char*>(map_) + p0 * page;
        const size_t len = std::min(size_, p1 * page) - p0 * page;
#ifdef MADV_POPULATE_READ
        if (::madvise(lo, len, MADV_POPULATE_READ) == 0) return;
#endif
        unsigned acc = 0;
        const volatile unsigned char* q = reinterpret_cast<const unsigned char*>(lo);
        for (size_t o = 0; o < len; o += page) acc += q[o];
        (void)acc;
    };
    std::vector<std::thread> pool;
    for (size_t i = 1; i < n; ++i) {
        try {
            pool.emplace_back(populate, i);
        } catch (...) {  // no more threads: this one does the rest
            for (size_t j = i; j < n; ++j) populate(j);
            break;
        }
    }
    populate(0);
    for (auto& t : pool) t.join();
}

}  // namespace vb
