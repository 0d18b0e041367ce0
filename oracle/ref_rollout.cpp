// Test-infrastructure driver around the UNMODIFIED reference host rollout (varda.cpp,
// src/varda/rollout.{h,cpp}) on the reference CPU fp32 backend. Compiled from the reference's own
// sources by oracle/Makefile into oracle/_ref/; never part of the product.
//
//   ref_rollout --model M.safetensors --input X.safetensors --steps N [--oldest] [--threads N]
//               [--out Y.safetensors]
//
// X holds "in.x" (1, T, G, V_in) and, for N > 1 with dynamic forcings, "forcings" (N - 1, G, F),
// replayed through RolloutRequest::replay_forcings (rollout.h:75-85). Runs varda::Rollout::run
// (rollout.cpp:116-155) with ConstantSource::Newest (default) or ::Oldest and writes every step's
// output as "y" (N, G, V_out) F32. Prints one JSON line with the per-step predict / update seconds.
#include <omp.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "varda/format.h"
#include "varda/rollout.h"
#include "varda/varda.h"

namespace {

[[noreturn]] void usage() {
    std::fprintf(stderr,
                 "usage: ref_rollout --model M --input X --steps N [--oldest] [--threads N] [--out Y]\n");
    std::exit(2);
}

}  // namespace

int main(int argc, char** argv) {
    std::string model_path, input_path, out_path;
    int steps = 1;
    bool oldest = false;
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
        else if (a == "--steps") steps = std::atoi(next().c_str());
        else if (a == "--oldest") oldest = true;
        else if (a == "--threads") opts.num_threads = std::atoi(next().c_str());
        else if (a == "--out") out_path = next();
        else usage();
    }
    if (model_path.empty() || input_path.empty() || steps < 1) usage();
    try {
        auto model = varda::Model::load(model_path, opts);
        const varda::Config& c = model->config();
        varda::SafeTensorsFile in(input_path);
        const varda::TensorView& x = in.take("in.x", varda::DType::F32,
                                             {1, c.n_input_steps, c.n_data_nodes, c.n_input_vars});
        varda::Rollout r(*model, oldest ? varda::ConstantSource::Oldest : varda::ConstantSource::Newest);
        const int F = r.update().F;
        const float* forcings = nullptr;
        if (steps > 1 && F > 0)
            forcings = in.take("forcings", varda::DType::F32, {steps - 1, c.n_data_nodes, F}).as<float>();

        const int64_t per = int64_t(c.n_data_nodes) * c.n_output_vars;
        std::vector<float> ys(size_t(per) * size_t(steps));
        varda::RolloutRequest q;
        q.x0 = x.as<float>();
        q.n_steps = steps;
        q.replay_forcings = forcings;
        q.on_step = [&](int s, const varda::DateTime&, const float* y) {
            std::memcpy(ys.data() + size_t(s) * size_t(per), y, size_t(per) * sizeof(float));
        };
        r.run(q);
        if (!out_path.empty())
            varda::write_safetensors(out_path, {{"y", varda::DType::F32, {steps, c.n_data_nodes, c.n_output_vars},
                                                 ys.data()}},
                                     {{"producer", "reference host rollout, cpu fp32 (oracle/_ref/ref_rollout)"}});
        std::printf("{\"threads\": %d, \"predict_s\": [", opts.num_threads > 0 ? opts.num_threads : omp_get_max_threads());
        for (int s = 0; s < steps; ++s) std::printf("%s%.6f", s ? ", " : "", r.times()[size_t(s)].predict);
        std::printf("], \"update_s\": [");
        for (int s = 0; s < steps; ++s) std::printf("%s%.6f", s ? ", " : "", r.times()[size_t(s)].update);
        std::printf("]}\n");
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ref_rollout: %s\n", e.what());
        return 1;
    }
    return 0;
}
