#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "common.h"
#include "json.h"

namespace vb {

namespace {
struct DT {
    DType t;
    const char* name;
    size_t size;
};
constexpr DT kTable[] = {{DType::F32, "F32", 4}, {DType::F16, "F16", 2}, {DType::BF16, "BF16", 2},
                         {DType::F64, "F64", 8}, {DType::I64, "I64", 8}, {DType::I32, "I32", 4},
                         {DType::I16, "I16", 2}, {DType::I8, "I8", 1},   {DType::U8, "U8", 1},
                         {DType::BOOL, "BOOL", 1}};
}  // namespace

const char* dtype_name(DType t) {
    for (const auto& d : kTable)
        if (d.t == t) return d.name;
    return "?";
}
size_t dtype_size(DType t) {
    for (const auto& d : kTable)
        if (d.t == t) return d.size;
    return 0;
}

std::string TensorView::shape_str() const {
    std::string s = "[";
    for (size_t i = 0; i < shape.size(); ++i) s += (i ? ", " : "") + std::to_string(shape[i]);
    return s + "]";
}

SafeTensorsFile::SafeTensorsFile(const std::string& path) : path_(path) {
    auto bad = [&](const std::string& m) { fail(kFormat, path + ": " + m); };
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) fail(kFormat, path + ": cannot open: " + std::strerror(errno));
    try {
        struct stat st {};
        if (::fstat(fd_, &st) != 0) bad("fstat failed");
        size_ = static_cast<size_t>(st.st_size);
        if (size_ < 8) bad("file too small for a safetensors header");
        map_ = ::mmap(nullptr, size_, PROT_READ, MAP_SHARED, fd_, 0);
        if (map_ == MAP_FAILED) {
            map_ = nullptr;
            bad("mmap failed");
        }
        const auto* base = static_cast<const char*>(map_);
        uint64_t n = 0;
        std::memcpy(&n, base, 8);
        if (n > size_ - 8) bad("header length exceeds file size");
        json::Value hdr = json::parse(base + 8, base + 8 + n);
        if (hdr.kind != json::Value::Object) bad("header is not a JSON object");
        const size_t data0 = 8 + n, data_size = size_ - data0;
        for (const auto& kv : hdr.obj) {
            if (kv.first == "__metadata__") {
                for (const auto& m : kv.second.obj) meta_[m.first] = m.second.as_str("metadata value");
                continue;
            }
            TensorView v;
            v.name = kv.first;
            const std::string& dt = kv.second.at("dtype").as_str("dtype");
            bool found = false;
            for (const auto& d : kTable)
                if (dt == d.name) v.dtype = d.t, found = true;
            if (!found) bad("unsupported dtype " + dt + " of " + v.name);
            v.shape = kv.second.at("shape").int64_list("shape");
            const auto off = kv.second.at("data_offsets").int64_list("data_offsets");
            if (off.size() != 2 || off[0] < 0 || off[0] > off[1] || uint64_t(off[1]) > data_size)
                bad("bad data_offsets for " + v.name);
            v.nbytes = size_t(off[1] - off[0]);
            uint64_t ne = 1;
            for (int64_t d : v.shape) {
                if (d < 0) bad("negative dimension in " + v.name);
                if (d != 0 && ne > UINT64_MAX / uint64_t(d)) bad("shape overflow in " + v.name);
                ne *= uint64_t(d);
            }
            if (ne * dtype_size(v.dtype) != v.nbytes) bad("size mismatch for " + v.name);
            v.data = base + data0 + off[0];
            if (reinterpret_cast<uintptr_t>(v.data) % dtype_size(v.dtype))
                bad("tensor " + v.name + " is not aligned to its element size");
            tensors_.emplace(v.name, std::move(v));
        }
    } catch (...) {
        if (map_) ::munmap(map_, size_);
        ::close(fd_);
        map_ = nullptr;
        fd_ = -1;
        throw;
    }
}

SafeTensorsFile::~SafeTensorsFile() {
    if (map_) ::munmap(map_, size_);
    if (fd_ >= 0) ::close(fd_);
}

std::string SafeTensorsFile::metadata(const std::string& key) const {
    auto it = meta_.find(key);
    if (it == meta_.end()) fail(kFormat, path_ + ": missing __metadata__ entry '" + key + "'");
    return it->second;
}

const TensorView& SafeTensorsFile::peek(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) fail(kFormat, path_ + ": missing tensor '" + name + "'");
    return it->second;
}

const TensorView& SafeTensorsFile::take(const std::string& name) {
    const TensorView& v = peek(name);
    consumed_.insert(name);
    return v;
}

const TensorView& SafeTensorsFile::take(const std::string& name, DType dtype, const std::vector<int64_t>& shape) {
    const TensorView& v = take(name);
    if (v.dtype != dtype)
        fail(kFormat, path_ + ": tensor '" + name + "' has dtype " + dtype_name(v.dtype) + ", expected " +
                          dtype_name(dtype));
    if (v.shape != shape) {
        TensorView w;
        w.shape = shape;
        fail(kFormat, path_ + ": tensor '" + name + "' has shape " + v.shape_str() + ", expected " + w.shape_str());
    }
    return v;
}

std::vector<std::string> SafeTensorsFile::names() const {
    std::vector<std::string> out;
    for (const auto& kv : tensors_) out.push_back(kv.first);
    return out;
}

std::vector<std::string> SafeTensorsFile::unconsumed() const {
    std::vector<std::string> out;
    for (const auto& kv : tensors_)
        if (!consumed_.count(kv.first)) out.push_back(kv.first);
    return out;
}

void SafeTensorsFile::require_all_consumed() const {
    auto left = unconsumed();
    if (left.empty()) return;
    std::string m = std::to_string(left.size()) + " tensor(s) not consumed by the engine:";
    for (size_t i = 0; i < left.size() && i < 20; ++i) m += " " + left[i];
    fail(kFormat, path_ + ": " + m);
}

void SafeTensorsFile::prefetch(int threads) const {
    if (const char* e = std::getenv("VB_PREFETCH_THREADS"); e && *e) threads = std::atoi(e);
    else if (threads <= 0) threads = 16;
    if (threads <= 0 || !map_) return;
    constexpr size_t kChunk = size_t(8) << 20;
    const size_t chunks = (size_ + kChunk - 1) / kChunk;
    threads = int(std::min<size_t>(size_t(threads), chunks));
    const size_t page = size_t(::sysconf(_SC_PAGESIZE));
    std::atomic<size_t> next{0};
    auto work = [&] {
        unsigned sum = 0;
        for (size_t c; (c = next.fetch_add(1)) < chunks;) {
            const size_t lo = c * kChunk, hi = std::min(size_, lo + kChunk);
            char* p = static_cast<char*>(map_) + lo;
#ifdef MADV_POPULATE_READ
            if (::madvise(p, hi - lo, MADV_POPULATE_READ) == 0) continue;
#endif
            const volatile unsigned char* q = reinterpret_cast<const unsigned char*>(p);
            for (size_t o = 0; o < hi - lo; o += page) sum += q[o];
        }
        (void)sum;
    };
    std::vector<std::thread> pool;
    for (int i = 1; i < threads; ++i) {
        try {
            pool.emplace_back(work);
        } catch (...) {
            break;
        }
    }
    work();
    for (auto& t : pool) t.join();
}

}  // namespace vb
