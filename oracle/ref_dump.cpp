// Test-infrastructure driver around the UNMODIFIED reference CPU fp32 backend (varda.cpp,
// src/varda/cpu/). It is compiled from the reference's own sources by oracle/Makefile into
// oracle/_ref/ and is never part of the product.
//
//   ref_dump --model M.safetensors --input X.safetensors [--key in.x] [--threads N]
//            [--steps N] [--dump OUT.safetensors] [--y-out Y.safetensors]
//
// Loads the model through the reference's public API (varda::Model::load, varda.h:37-50), runs
// predict_step (model.cpp:431) `--steps` times without a hook and prints one JSON line with the
// load time and the per-step wall times. With --dump it first runs one hooked predict_step and
// writes every contract activation (docs/format.md section 2 of the reference) as F32 into
// OUT.safetensors with varda::write_safetensors (format.h:82), so tests can compare against the
// reference's own numbers. With --y-out it writes the last step's output y (F32, the predict_step
// output shape) alone, which is all a full-size model needs kept (its activations run to many GB).
#include <omp.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "varda/format.h"
#include "varda/varda.h"

namespace {

double now_s() {
    using namespace std::chrono;
    return duration<double>(steady_clock::now().time_since_epoch()).count();
}

[[noreturn]] void usage() {
    std::fprintf(stderr,
                 "usage: ref_dump --model M --input X [--key in.x] [--threads N] [--steps N] [--dump OUT] "
                 "[--y-out Y]\n");
    std::exit(2);
}

}  // namespace

int main(int argc, char** argv) {
    std::string model_path, input_path, key = "in.x", dump_path, y_path;
    int steps = 1;
    varda::Options opts;
    opts.device = varda::Device::CPU;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        auto next = [&]() -> std::string {
            if (i + 1 >= argc) usage();
            return argv[++i];
        };
        if (a == "--model") model_path = next();
        else if (a == "--input") input_path = next();
        else if (a == "--key") key = next();
        else if (a == "--threads") opts.num_threads = std::atoi(next().c_str());
        else if (a == "--steps") steps = std::atoi(next().c_str());
        else if (a == "--dump") dump_path = next();
        else if (a == "--y-out") y_path = next();
        else usage();
    }
    if (model_path.empty() || input_path.empty()) usage();
    try {
        const double t0 = now_s();
        auto model = varda::Model::load(model_path, opts);
        const double t_load = now_s() - t0;
        const varda::Config& c = model->config();
        varda::SafeTensorsFile in(input_path);
        const varda::TensorView& x = in.take(key, varda::DType::F32,
                                             {1, c.n_input_steps, c.n_data_nodes, c.n_input_vars});
        const int64_t n_out = int64_t(c.n_output_steps) * c.n_data_nodes * c.n_output_vars;
        std::vector<float> y(static_cast<size_t>(n_out));

        if (!dump_path.empty()) {
            // Keep every activation (host fp32) until the end, then write one file.
            std::map<std::string, std::pair<std::vector<int64_t>, std::vector<float>>> acts;
            std::vector<std::string> order;
            varda::ActivationHook hook = [&](const std::string& k, const float* d, const std::vector<int64_t>& s) {
                int64_t n = 1;
                for (int64_t v : s) n *= v;
                acts[k] = {s, std::vector<float>(d, d + n)};
                order.push_back(k);
            };
            model->predict_step(x.as<float>(), y.data(), &hook);
            std::vector<varda::TensorOut> outs;
            for (const auto& k : order)
                outs.push_back({k, varda::DType::F32, acts[k].first, acts[k].second.data()});
            varda::write_safetensors(dump_path, outs, {{"producer", "reference cpu fp32 (oracle/_ref/ref_dump)"}});
        }

        std::vector<double> times;
        for (int s = 0; s < steps; ++s) {
            const double t1 = now_s();
            model->predict_step(x.as<float>(), y.data(), nullptr);
            times.push_back(now_s() - t1);
        }
        if (!y_path.empty())
            varda::write_safetensors(y_path,
                                     {{"y", varda::DType::F32,
                                       {1, c.n_output_steps, 1, c.n_data_nodes, c.n_output_vars}, y.data()}},
                                     {{"producer", "reference cpu fp32 (oracle/_ref/ref_dump)"}});
        double sum = 0;
        for (float v : y) sum += v;
        std::printf("{\"load_s\": %.4f, \"threads\": %d, \"steps_s\": [", t_load,
                    opts.num_threads > 0 ? opts.num_threads : omp_get_max_threads());
        for (size_t i = 0; i < times.size(); ++i) std::printf("%s%.6f", i ? ", " : "", times[i]);
        std::printf("], \"y_sum\": %.9g}\n", sum);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ref_dump: %s\n", e.what());
        return 1;
    }
    return 0;
}
