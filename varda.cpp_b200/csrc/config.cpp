#include "config.h"

#include <algorithm>

#include "common.h"
#include "json.h"

namespace vb {

namespace {
[[noreturn]] void unsupported(const std::string& what) { fail(kFormat, "unsupported config: " + what); }
void require(bool ok, const std::string& what) {
    if (!ok) fail(kFormat, "inconsistent config: " + what);
}
void check_range(const std::vector<int>& idx, int n, const std::string& what) {
    for (int i : idx) require(i >= 0 && i < n, what + " index " + std::to_string(i) + " out of range");
}
}  // namespace

bool Config::is_absent(const std::string& name) const {
    return std::find(absent.begin(), absent.end(), name) != absent.end();
}

Config parse_config(const std::string& text) {
    const json::Value j = json::parse(text);
    Config c;
    c.json_text = text;
    c.format_version = int(j.at("format_version").as_int("format_version"));
    if (c.format_version != 3)
        unsupported("format_version " + std::to_string(c.format_version) + " (this engine reads 3)");
    const json::Value& src = j.at("source");
    if (src.has("uuid") && src.at("uuid").kind == json::Value::String) c.uuid = src.at("uuid").str;

    const json::Value& arch = j.at("architecture");
    auto want = [&](const char* part, const char* kind) {
        const std::string& k = arch.at(part).at("kind").as_str("kind");
        if (k != kind) unsupported(std::string("architecture.") + part + ".kind '" + k + "'");
    };
    c.model_kind = arch.at("model").at("kind").as_str("kind");
    if (c.model_kind != "enc_proc_dec" && c.model_kind != "enc_proc_dec_interpolator")
        unsupported("architecture.model.kind '" + c.model_kind + "'");
    want("encoder", "graph_transformer_forward_mapper");
    want("processor", "graph_transformer_processor");
    want("decoder", "graph_transformer_backward_mapper");

    const json::Value& d = j.at("dims");
    auto I = [&](const char* k) { return int(d.at(k).as_int(k)); };
    c.num_channels = I("num_channels");
    c.num_heads = I("num_heads");
    c.head_dim = I("head_dim");
    c.mlp_hidden = I("mlp_hidden");
    c.num_processor_layers = I("num_processor_layers");
    c.n_input_steps = I("n_input_steps");
    c.n_output_steps = d.has("n_output_steps") ? I("n_output_steps") : 1;
    c.n_data_vars = I("n_data_vars");
    c.n_input_vars = I("n_input_vars");
    c.n_output_vars = I("n_output_vars");
    c.n_data_nodes = d.at("n_data_nodes").as_int("n_data_nodes");
    c.n_hidden_nodes = d.at("n_hidden_nodes").as_int("n_hidden_nodes");
    c.node_attr_dim = I("node_attr_dim");
    c.edge_attr_dim = I("edge_attr_dim");
    c.layer_norm_eps = float(d.at("layer_norm_eps").as_num("layer_norm_eps"));
    const std::string& gelu = d.at("gelu_approximate").as_str("gelu_approximate");
    if (gelu == "none") c.gelu_tanh = false;
    else if (gelu == "tanh") c.gelu_tanh = true;
    else unsupported("dims.gelu_approximate '" + gelu + "'");
    c.latent_skip = d.at("latent_skip").as_bool("latent_skip");

    require(c.num_heads * c.head_dim == c.num_channels, "num_heads * head_dim != num_channels");
    require(c.num_channels > 0 && c.num_heads > 0 && c.mlp_hidden > 0, "non-positive width");
    require(c.num_processor_layers >= 0 && c.n_input_steps >= 1, "layer/step counts");
    require(c.n_data_vars > 0 && c.n_input_vars > 0 && c.n_output_vars > 0, "variable counts");
    require(c.n_data_nodes > 0 && c.n_hidden_nodes > 0, "node counts");
    require(c.node_attr_dim >= 1 && c.edge_attr_dim >= 1, "node_attr_dim and edge_attr_dim must be >= 1");
    require(c.layer_norm_eps > 0.0f, "layer_norm_eps");
    if (c.is_interpolator()) {
        require(c.n_output_steps >= 1, "n_output_steps");
        const json::Value& t = j.at("times");
        c.input_times = t.at("input").int_list("times.input");
        c.output_times = t.at("target").int_list("times.target");
        c.frequency_hours = int(t.at("frequency_hours").as_int("frequency_hours"));
        require(int(c.input_times.size()) == c.n_input_steps, "times.input size != n_input_steps");
        require(int(c.output_times.size()) == c.n_output_steps, "times.target size != n_output_steps");
        require(c.frequency_hours >= 1, "times.frequency_hours");
        for (size_t i = 1; i < c.input_times.size(); ++i)
            require(c.input_times[i] > c.input_times[i - 1], "times.input not increasing");
        for (size_t i = 1; i < c.output_times.size(); ++i)
            require(c.output_times[i] > c.output_times[i - 1], "times.target not increasing");
    } else if (c.n_output_steps != 1) {
        unsupported("n_output_steps != 1 for a forecaster");
    }

    const json::Value& v = j.at("variables");
    c.var_data = v.at("data").str_list("variables.data");
    c.var_input = v.at("input").str_list("variables.input");
    c.var_output = v.at("output").str_list("variables.output");
    require(int(c.var_data.size()) == c.n_data_vars, "variables.data size");
    require(int(c.var_input.size()) == c.n_input_vars, "variables.input size");
    require(int(c.var_output.size()) == c.n_output_vars, "variables.output size");

    const json::Value& ix = j.at("indices");
    c.norm_input = ix.at("norm_input").int_list("norm_input");
    c.norm_output = ix.at("norm_output").int_list("norm_output");
    c.residual_input = ix.at("residual_input").int_list("residual_input");
    c.residual_output = ix.at("residual_output").int_list("residual_output");
    require(int(c.norm_input.size()) == c.n_input_vars, "indices.norm_input size");
    require(int(c.norm_output.size()) == c.n_output_vars, "indices.norm_output size");
    require(c.residual_input.size() == c.residual_output.size(), "residual index sizes differ");
    check_range(c.norm_input, c.n_data_vars, "norm_input");
    check_range(c.norm_output, c.n_data_vars, "norm_output");
    check_range(c.residual_input, c.n_input_vars, "residual_input");
    check_range(c.residual_output, c.n_output_vars, "residual_output");

    const json::Value& r = j.at("residual");
    if (r.at("type").as_str("residual.type") != "skip") unsupported("residual.type '" + r.at("type").str + "'");
    c.residual_step = int(r.at("step").as_int("residual.step"));
    if (c.residual_step < 0) c.residual_step += c.n_input_steps;
    require(c.residual_step >= 0 && c.residual_step < c.n_input_steps, "residual.step");

    for (const json::Value& b : j.at("bounding").arr) {
        Bounding bd;
        bd.type = b.at("type").as_str("bounding.type");
        bd.index = b.at("index").int_list("bounding.index");
        check_range(bd.index, c.n_output_vars, "bounding");
        if (bd.type == "relu") {
        } else if (bd.type == "hardtanh" || bd.type == "fraction") {
            bd.min = float(b.at("min").as_num("bounding.min"));
            bd.max = float(b.at("max").as_num("bounding.max"));
            if (bd.type == "fraction") {
                bd.total_index = b.at("total_index").int_list("bounding.total_index");
                check_range(bd.total_index, c.n_output_vars, "bounding total_index");
                require(bd.total_index.size() == 1 || bd.total_index.size() == bd.index.size(),
                        "fraction total_index size");
            }
        } else {
            unsupported("bounding type '" + bd.type + "'");
        }
        c.bounding.push_back(bd);
    }

    const json::Value& blocks = j.at("blocks");
    std::vector<std::string> order{"enc.block"};
    for (int i = 0; i < c.num_processor_layers; ++i) order.push_back("proc." + std::to_string(i));
    order.push_back("dec.block");
    require(blocks.size() == order.size(), "blocks count");
    for (const auto& name : order) {
        const std::string& kind = blocks.at(name).at("kind").as_str("block kind");
        const bool mapper = name == "enc.block" || name == "dec.block";
        const char* want_kind = mapper ? "graph_transformer_mapper_block" : "graph_transformer_processor_block";
        if (kind != want_kind) unsupported("block " + name + " kind '" + kind + "'");
        c.block_names.push_back(name);
    }
    if (j.has("absent")) c.absent = j.at("absent").str_list("absent");

    if (j.has("forcings")) {
        const json::Value& f = j.at("forcings");
        c.has_forcings = true;
        const auto dyn = f.at("dynamic").str_list("forcings.dynamic");
        const auto con = f.at("constant").str_list("forcings.constant");
        c.forcing_dynamic_index = f.at("dynamic_input_index").int_list("forcings.dynamic_input_index");
        c.forcing_constant_index = f.at("constant_input_index").int_list("forcings.constant_input_index");
        require(dyn.size() == c.forcing_dynamic_index.size(), "forcings.dynamic sizes");
        require(con.size() == c.forcing_constant_index.size(), "forcings.constant sizes");
        check_range(c.forcing_dynamic_index, c.n_input_vars, "forcings.dynamic_input_index");
        check_range(c.forcing_constant_index, c.n_input_vars, "forcings.constant_input_index");
        for (size_t i = 0; i < dyn.size(); ++i)
            require(c.var_input[c.forcing_dynamic_index[i]] == dyn[i], "forcings.dynamic name/index");
        for (size_t i = 0; i < con.size(); ++i)
            require(c.var_input[c.forcing_constant_index[i]] == con[i], "forcings.constant name/index");
        if (f.has("timestep_hours")) c.timestep_hours = int(f.at("timestep_hours").as_int("timestep_hours"));
    }
    if (j.has("timestep_hours") && !c.timestep_hours) c.timestep_hours = int(j.at("timestep_hours").as_int());
    return c;
}

}  // namespace vb
