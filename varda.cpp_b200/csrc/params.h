// The GraphTransformer's parameters on the device, in the layouts the kernels read, and the schema of
// a format v3 model file's tensors (names, dtypes, shapes) that both validates a file before any
// device work and drives the upload.
//
// Layouts:
//   Dense<T>   a Linear y = x W^T + b, or several Linears with the same input stacked by output rows
//              (the processor's q|k|v|self, the mappers' q|self and k|v), stored as T with the input
//              dimension padded to a multiple of 8 elements (16-byte rows for the tensor-memory-access
//              loads of the GEMM), zero padded; the bias as T (absent biases: no bias buffer when none
//              of the stacked Linears has one, zeros for the ones that lack it).
//   Affine     a LayerNorm's weight and bias, fp32.
//   edge fold  fp32 [4, C]: the edge Linear's weight columns (attribute-major, zero padded to three
//              attributes), then its bias, so the attention kernels read per lane contiguous channels of
//              each; in fp16 mode rounded to fp16 values, as autocast runs the edge Linear in fp16.
#pragma once

#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "common.h"
#include "config.h"
#include "safetensors.h"

namespace vb {

template <class T> struct Dense {
    DeviceBuffer weight, bias;
    DeviceBuffer colsum;  // fp32 [out]: set when a LayerNorm is folded into the weights (fold_layernorm)
    int64_t out = 0, in = 0, ld_in = 0;
    const T* w() const { return weight.as<T>(); }
    const T* b() const { return bias.get() ? bias.as<T>() : nullptr; }
    const float* cs() const { return colsum.get() ? colsum.as<float>() : nullptr; }
};

struct Affine {
    DeviceBuffer gamma, beta;
    const float* g() const { return gamma.as<float>(); }
    const float* b() const { return beta.get() ? beta.as<float>() : nullptr; }
};

// One graph-transformer block. Processor blocks project their destination rows to q|k|v|self in one
// product (proj_qkvx); the mappers project destinations to q|self (proj_qx) and sources to k|v
// (proj_kv), with their own source LayerNorm.
template <class T> struct AttnLayer {
    bool mapper = false;
    Affine norm_src, norm_dst, norm_ffn;
    Dense<T> proj_qkvx, proj_qx, proj_kv, proj_out, ffn_up, ffn_down;
    DeviceBuffer edge_fold;
};

struct TensorSpec {
    std::string name;
    DType dtype;
    std::vector<int64_t> shape;  // -1: any length (edge counts)
};

// Every tensor a model file of config `c` holds (config `absent` biases left out), in a fixed order.
std::vector<TensorSpec> model_schema(const Config& c);
// Checks the file against the schema: every tensor present with its dtype and shape, nothing else
// except the optional grid.latitudes / grid.longitudes pair. kFormat errors; no device work.
void validate_model_file(const SafeTensorsFile& f, const Config& c);

// f(begin, end) over [0, n) on up to 16 host threads, about `grain` items or more each; f must not
// depend on how [0, n) is split.
template <class F> void split_work(int64_t n, int64_t grain, F f) {
    const int64_t hw = std::max<int64_t>(1, int64_t(std::thread::hardware_concurrency()));
    const int64_t nt = std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(hw, 16), n / std::max<int64_t>(grain, 1)));
    if (nt == 1) return f(int64_t(0), n);
    std::vector<std::thread> pool;
    for (int64_t i = 1; i < nt; ++i) pool.emplace_back(f, n * i / nt, n * (i + 1) / nt);
    f(int64_t(0), n / nt);
    for (auto& t : pool) t.join();
}

// Reads parameters out of the model file (marking them consumed) and uploads them to the current
// device; counts the bytes uploaded into `uploaded`.
template <class T> class ParamLoader {
public:
    ParamLoader(SafeTensorsFile& f, const Config& c, size_t& uploaded) : f_(f), c_(c), uploaded_(uploaded) {}

    // The Linears `names` (each [rows_each, in]) stacked by output rows.
    Dense<T> dense(const std::vector<std::string>& names, int64_t rows_each, int64_t in) {
        Dense<T> d;
        d.in = in, d.ld_in = (in + 7) / 8 * 8, d.out = rows_each * int64_t(names.size());
        std::vector<T> w(size_t(d.out * d.ld_in), T(0.0f)), b(size_t(d.out), T(0.0f));
        bool has_bias = false;
        for (size_t i = 0; i < names.size(); ++i) {
            const float* src = f_.take(names[i] + ".weight", DType::F32, {rows_each, in}).template as<float>();
            T* dst = w.data() + i * size_t(rows_each * d.ld_in);
            const int64_t ld = d.ld_in;
            split_work(rows_each, std::max<int64_t>(1, (int64_t(1) << 20) / std::max<int64_t>(in, 1)),
                       [&](int64_t r0, int64_t r1) {
                           for (int64_t r = r0; r < r1; ++r) {
                               const float* s = src + r * in;
                               T* o = dst + r * ld;
                               for (int64_t k = 0; k < in; ++k) o[k] = T(s[k]);
                           }
                       });
            if (c_.is_absent(names[i] + ".bias")) continue;
            const float* bs = f_.take(names[i] + ".bias", DType::F32, {rows_each}).template as<float>();
            for (int64_t r = 0; r < rows_each; ++r) b[i * size_t(rows_each) + size_t(r)] = T(bs[r]);
            has_bias = true;
        }
        d.weight = put(w.data(), w.size() * sizeof(T));
        if (has_bias) d.bias = put(b.data(), b.size() * sizeof(T));
        return d;
    }

    Affine affine(const std::string& name, int64_t width) {
        Affine a;
        const TensorView& g = f_.take(name + ".weight", DType::F32, {width});
        a.gamma = put(g.data, g.nbytes);
        if (!c_.is_absent(name + ".bias")) {
            const TensorView& b = f_.take(name + ".bias", DType::F32, {width});
            a.beta = put(b.data, b.nbytes);
        }
        return a;
    }

    DeviceBuffer edge_fold(const std::string& name, int64_t width) {
        const int A = c_.edge_attr_dim;
        const float* w = f_.take(name + ".weight", DType::F32, {width, A}).template as<float>();
        std::vector<float> fold(size_t(4 * width), 0.0f);
        for (int a = 0; a < A; ++a)
            for (int64_t ch = 0; ch < width; ++ch) fold[size_t(a * width + ch)] = storage(w[ch * A + a]);
        if (!c_.is_absent(name + ".bias")) {
            const float* b = f_.take(name + ".bias", DType::F32, {width}).template as<float>();
            for (int64_t ch = 0; ch < width; ++ch) fold[size_t(3 * width + ch)] = storage(b[ch]);
        }
        return put(fold.data(), fold.size() * sizeof(float));
    }

    AttnLayer<T> layer(const std::string& prefix, bool mapper, int64_t C, int64_t mlp) {
        auto n = [&](const char* part) { return prefix + "." + part; };
        AttnLayer<T> l;
        l.mapper = mapper;
        if (mapper) l.norm_src = affine(n("ln_src"), C);
        l.norm_dst = affine(n("ln_dst"), C);
        l.norm_ffn = affine(n("ln_mlp"), C);
        if (mapper) {
            l.proj_qx = dense({n("q"), n("self")}, C, C);
            l.proj_kv = dense({n("k"), n("v")}, C, C);
        } else {
            l.proj_qkvx = dense({n("q"), n("k"), n("v"), n("self")}, C, C);
        }
        l.proj_out = dense({n("proj")}, C, C);
        l.ffn_up = dense({n("mlp1")}, mlp, C);
        l.ffn_down = dense({n("mlp2")}, C, mlp);
        l.edge_fold = edge_fold(n("edge"), C);
        return l;
    }

private:
    // the value the engine computes with: the fp32 value, or its fp16 rounding in fp16 mode
    static float storage(float x) { return std::is_same<T, float>::value ? x : __half2float(__float2half_rn(x)); }
    DeviceBuffer put(const void* host, size_t bytes) {
        DeviceBuffer d(bytes);
        if (bytes) VB_CUDA(cudaMemcpy(d.get(), host, bytes, cudaMemcpyHostToDevice));
        uploaded_ += bytes;
        return d;
    }
    SafeTensorsFile& f_;
    const Config& c_;
    size_t& uploaded_;
};

}  // namespace vb
