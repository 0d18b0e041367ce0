// Model configuration from the `config` metadata JSON (format v3) of a converted varda.cpp model:
// the fields of the reference's varda::Config (src/varda/config.h:11-77) that this engine uses, read
// and validated against the format contract (the reference's docs/format.md section 1.2) by
// config.cpp; unknown kinds and variants are rejected at load (kFormat errors).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace vb {

struct Bounding {
    std::string type;  // "relu" | "hardtanh" | "fraction"
    std::vector<int> index, total_index;
    float min = 0.0f, max = 0.0f;
};

struct Config {
    std::string json_text;
    int format_version = 0;
    std::string uuid;
    std::string model_kind;  // "enc_proc_dec" | "enc_proc_dec_interpolator"
    int num_channels = 0, num_heads = 0, head_dim = 0, mlp_hidden = 0;
    int num_processor_layers = 0, n_input_steps = 0, n_output_steps = 1;
    int n_data_vars = 0, n_input_vars = 0, n_output_vars = 0;
    int64_t n_data_nodes = 0, n_hidden_nodes = 0;
    int node_attr_dim = 0, edge_attr_dim = 0;
    float layer_norm_eps = 0.0f;
    bool gelu_tanh = false, latent_skip = false;
    std::vector<int> input_times, output_times;
    int frequency_hours = 0;
    std::vector<std::string> var_data, var_input, var_output;
    std::vector<int> norm_input, norm_output, residual_input, residual_output;
    int residual_step = -1;
    std::vector<Bounding> bounding;
    std::vector<std::string> block_names;  // enc.block, proc.0 .. proc.{n-1}, dec.block
    std::vector<std::string> absent;
    bool has_forcings = false;
    std::vector<int> forcing_dynamic_index, forcing_constant_index;
    int timestep_hours = 0;

    int src_features() const { return n_input_steps * n_input_vars + node_attr_dim; }
    int dec_out_features() const { return n_output_steps * n_output_vars; }
    bool is_interpolator() const { return model_kind == "enc_proc_dec_interpolator"; }
    bool is_absent(const std::string& name) const;
};

Config parse_config(const std::string& json_text);

}  // namespace vb
