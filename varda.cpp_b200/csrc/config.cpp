// Reader of the `config` metadata of a converted model file: the format v3 contract of varda.cpp
// (docs/format.md section 1.2 of the reference: keys format_version, source, architecture, dims,
// variables, indices, residual, bounding, blocks, absent, optional times and forcings).
//
// Table-driven. Scalar fields are rows of a schema (JSON path, type, required or defaulted, where the
// value goes) read by one loop; enumerated fields list their accepted values; the relations between
// fields are a table of named predicates checked once everything is read. The structured sections
// (bounding list, blocks, interpolator times, forcings) have a reader each. Every problem is a
// kFormat error that names the JSON path involved; an unknown kind or variant is refused at load.
#include "config.h"

#include <algorithm>
#include <functional>

#include "common.h"
#include "json.h"

namespace vb {

namespace {

[[noreturn]] void bad(const std::string& msg) { fail(kFormat, "model config: " + msg); }

// The value at a dotted path ("dims.num_heads"), or nullptr when a component is missing.
const json::Value* find(const json::Value& root, const std::string& path) {
    const json::Value* v = &root;
    size_t b = 0;
    while (b <= path.size()) {
        size_t e = path.find('.', b);
        if (e == std::string::npos) e = path.size();
        const std::string key = path.substr(b, e - b);
        if (!v->has(key)) return nullptr;
        v = &v->at(key);
        b = e + 1;
    }
    return v;
}
const json::Value& need(const json::Value& root, const std::string& path) {
    const json::Value* v = find(root, path);
    if (!v) bad(path + " is missing");
    return *v;
}

int64_t int_of(const json::Value& v, const std::string& path) {
    if (v.kind != json::Value::Number) bad(path + " must be a number");
    if (v.is_int) return v.inum;
    if (v.num != double(int64_t(v.num))) bad(path + " must be an integer");
    return int64_t(v.num);
}
std::vector<int> ints_of(const json::Value& v, const std::string& path) {
    if (v.kind != json::Value::Array) bad(path + " must be a list");
    std::vector<int> out;
    for (size_t i = 0; i < v.arr.size(); ++i) out.push_back(int(int_of(v.arr[i], path + "[" + std::to_string(i) + "]")));
    return out;
}
std::vector<std::string> strs_of(const json::Value& v, const std::string& path) {
    if (v.kind != json::Value::Array) bad(path + " must be a list");
    std::vector<std::string> out;
    for (const auto& e : v.arr) {
        if (e.kind != json::Value::String) bad(path + " must list strings");
        out.push_back(e.str);
    }
    return out;
}
const std::string& str_of(const json::Value& v, const std::string& path) {
    if (v.kind != json::Value::String) bad(path + " must be a string");
    return v.str;
}

// ---- scalar schema
enum class Kind { Int, Int64, Float, Bool };
struct Scalar {
    const char* path;
    Kind kind;
    bool required;
    double dflt;                          // used when not required and absent
    std::function<void(Config&, double)> set;
};
// ---- enumerated strings: the accepted values and what each one means
struct Choice {
    const char* path;
    std::vector<const char*> accepted;
    std::function<void(Config&, const std::string&)> set;
};
// ---- relations checked after reading
struct Rule {
    const char* what;
    std::function<bool(const Config&)> holds;
};

const std::vector<Scalar>& scalar_schema() {
    static const std::vector<Scalar> s = {
        {"format_version", Kind::Int, true, 0, [](Config& c, double v) { c.format_version = int(v); }},
        {"dims.num_channels", Kind::Int, true, 0, [](Config& c, double v) { c.num_channels = int(v); }},
        {"dims.num_heads", Kind::Int, true, 0, [](Config& c, double v) { c.num_heads = int(v); }},
        {"dims.head_dim", Kind::Int, true, 0, [](Config& c, double v) { c.head_dim = int(v); }},
        {"dims.mlp_hidden", Kind::Int, true, 0, [](Config& c, double v) { c.mlp_hidden = int(v); }},
        {"dims.num_processor_layers", Kind::Int, true, 0, [](Config& c, double v) { c.num_processor_layers = int(v); }},
        {"dims.n_input_steps", Kind::Int, true, 0, [](Config& c, double v) { c.n_input_steps = int(v); }},
        {"dims.n_output_steps", Kind::Int, false, 1, [](Config& c, double v) { c.n_output_steps = int(v); }},
        {"dims.n_data_vars", Kind::Int, true, 0, [](Config& c, double v) { c.n_data_vars = int(v); }},
        {"dims.n_input_vars", Kind::Int, true, 0, [](Config& c, double v) { c.n_input_vars = int(v); }},
        {"dims.n_output_vars", Kind::Int, true, 0, [](Config& c, double v) { c.n_output_vars = int(v); }},
        {"dims.n_data_nodes", Kind::Int64, true, 0, [](Config& c, double v) { c.n_data_nodes = int64_t(v); }},
        {"dims.n_hidden_nodes", Kind::Int64, true, 0, [](Config& c, double v) { c.n_hidden_nodes = int64_t(v); }},
        {"dims.node_attr_dim", Kind::Int, true, 0, [](Config& c, double v) { c.node_attr_dim = int(v); }},
        {"dims.edge_attr_dim", Kind::Int, true, 0, [](Config& c, double v) { c.edge_attr_dim = int(v); }},
        {"dims.layer_norm_eps", Kind::Float, true, 0, [](Config& c, double v) { c.layer_norm_eps = float(v); }},
        {"dims.latent_skip", Kind::Bool, true, 0, [](Config& c, double v) { c.latent_skip = v != 0; }},
        {"residual.step", Kind::Int, true, 0, [](Config& c, double v) { c.residual_step = int(v); }},
    };
    return s;
}

const std::vector<Choice>& choice_schema() {
    static const std::vector<Choice> s = {
        {"architecture.model.kind", {"enc_proc_dec", "enc_proc_dec_interpolator"},
         [](Config& c, const std::string& v) { c.model_kind = v; }},
        {"architecture.encoder.kind", {"graph_transformer_forward_mapper"}, nullptr},
        {"architecture.processor.kind", {"graph_transformer_processor"}, nullptr},
        {"architecture.decoder.kind", {"graph_transformer_backward_mapper"}, nullptr},
        {"dims.gelu_approximate", {"none", "tanh"}, [](Config& c, const std::string& v) { c.gelu_tanh = v == "tanh"; }},
        {"residual.type", {"skip"}, nullptr},
    };
    return s;
}

bool all_in(const std::vector<int>& idx, int n) {
    return std::all_of(idx.begin(), idx.end(), [n](int i) { return i >= 0 && i < n; });
}
bool increasing(const std::vector<int>& v) {
    for (size_t i = 1; i < v.size(); ++i)
        if (v[i] <= v[i - 1]) return false;
    return true;
}

const std::vector<Rule>& rules() {
    static const std::vector<Rule> r = {
        {"format_version == 3 (the only version this engine reads)", [](const Config& c) { return c.format_version == 3; }},
        {"dims.num_heads * dims.head_dim == dims.num_channels",
         [](const Config& c) { return c.num_heads * c.head_dim == c.num_channels; }},
        {"dims.num_channels, num_heads, mlp_hidden > 0",
         [](const Config& c) { return c.num_channels > 0 && c.num_heads > 0 && c.mlp_hidden > 0; }},
        {"dims.num_processor_layers >= 0 and dims.n_input_steps >= 1",
         [](const Config& c) { return c.num_processor_layers >= 0 && c.n_input_steps >= 1; }},
        {"dims.n_data_vars, n_input_vars, n_output_vars > 0",
         [](const Config& c) { return c.n_data_vars > 0 && c.n_input_vars > 0 && c.n_output_vars > 0; }},
        {"dims.n_data_nodes, n_hidden_nodes > 0", [](const Config& c) { return c.n_data_nodes > 0 && c.n_hidden_nodes > 0; }},
        {"dims.node_attr_dim, edge_attr_dim >= 1", [](const Config& c) { return c.node_attr_dim >= 1 && c.edge_attr_dim >= 1; }},
        {"dims.layer_norm_eps > 0", [](const Config& c) { return c.layer_norm_eps > 0.0f; }},
        {"dims.n_output_steps == 1 for a forecaster (enc_proc_dec)",
         [](const Config& c) { return c.is_interpolator() ? c.n_output_steps >= 1 : c.n_output_steps == 1; }},
        {"variables.data / input / output sizes == dims.n_data_vars / n_input_vars / n_output_vars",
         [](const Config& c) {
             return int(c.var_data.size()) == c.n_data_vars && int(c.var_input.size()) == c.n_input_vars &&
                    int(c.var_output.size()) == c.n_output_vars;
         }},
        {"indices.norm_input: one data-variable index per input variable",
         [](const Config& c) { return int(c.norm_input.size()) == c.n_input_vars && all_in(c.norm_input, c.n_data_vars); }},
        {"indices.norm_output: one data-variable index per output variable",
         [](const Config& c) { return int(c.norm_output.size()) == c.n_output_vars && all_in(c.norm_output, c.n_data_vars); }},
        {"indices.residual_input / residual_output: pairs of an input and an output variable",
         [](const Config& c) {
             return c.residual_input.size() == c.residual_output.size() && all_in(c.residual_input, c.n_input_vars) &&
                    all_in(c.residual_output, c.n_output_vars);
         }},
        {"residual.step selects an input step (negative: from the last)",
         [](const Config& c) { return c.residual_step >= 0 && c.residual_step < c.n_input_steps; }},
        {"times (interpolator): one increasing index per input and output step, frequency_hours >= 1",
         [](const Config& c) {
             if (!c.is_interpolator()) return true;
             return int(c.input_times.size()) == c.n_input_steps && int(c.output_times.size()) == c.n_output_steps &&
                    c.frequency_hours >= 1 && increasing(c.input_times) && increasing(c.output_times);
         }},
    };
    return r;
}

void read_scalars(const json::Value& root, Config& c) {
    for (const Scalar& f : scalar_schema()) {
        const json::Value* v = find(root, f.path);
        if (!v) {
            if (f.required) bad(std::string(f.path) + " is missing");
            f.set(c, f.dflt);
            continue;
        }
        switch (f.kind) {
            case Kind::Int:
            case Kind::Int64: f.set(c, double(int_of(*v, f.path))); break;
            case Kind::Float:
                if (v->kind != json::Value::Number) bad(std::string(f.path) + " must be a number");
                f.set(c, v->is_int ? double(v->inum) : v->num);
                break;
            case Kind::Bool:
                if (v->kind != json::Value::Bool) bad(std::string(f.path) + " must be true or false");
                f.set(c, v->b ? 1.0 : 0.0);
                break;
        }
    }
    // 64-bit node counts are read exactly (not through the double above)
    c.n_data_nodes = int_of(need(root, "dims.n_data_nodes"), "dims.n_data_nodes");
    c.n_hidden_nodes = int_of(need(root, "dims.n_hidden_nodes"), "dims.n_hidden_nodes");
}

void read_choices(const json::Value& root, Config& c) {
    for (const Choice& f : choice_schema()) {
        const std::string& v = str_of(need(root, f.path), f.path);
        const bool ok = std::any_of(f.accepted.begin(), f.accepted.end(), [&](const char* a) { return v == a; });
        if (!ok) {
            std::string list;
            for (const char* a : f.accepted) list += std::string(list.empty() ? "" : ", ") + a;
            bad(std::string(f.path) + " = '" + v + "' is not supported (accepted: " + list + ")");
        }
        if (f.set) f.set(c, v);
    }
}

void read_lists(const json::Value& root, Config& c) {
    c.var_data = strs_of(need(root, "variables.data"), "variables.data");
    c.var_input = strs_of(need(root, "variables.input"), "variables.input");
    c.var_output = strs_of(need(root, "variables.output"), "variables.output");
    c.norm_input = ints_of(need(root, "indices.norm_input"), "indices.norm_input");
    c.norm_output = ints_of(need(root, "indices.norm_output"), "indices.norm_output");
    c.residual_input = ints_of(need(root, "indices.residual_input"), "indices.residual_input");
    c.residual_output = ints_of(need(root, "indices.residual_output"), "indices.residual_output");
    if (const json::Value* a = find(root, "absent")) c.absent = strs_of(*a, "absent");
    if (const json::Value* u = find(root, "source.uuid"); u && u->kind == json::Value::String) c.uuid = u->str;
    if (c.is_interpolator()) {
        c.input_times = ints_of(need(root, "times.input"), "times.input");
        c.output_times = ints_of(need(root, "times.target"), "times.target");
        c.frequency_hours = int(int_of(need(root, "times.frequency_hours"), "times.frequency_hours"));
    }
}

// bounding: a list of {type, index[, min, max][, total_index]} applied in order
void read_bounding(const json::Value& root, Config& c) {
    const json::Value& list = need(root, "bounding");
    if (list.kind != json::Value::Array) bad("bounding must be a list");
    for (size_t i = 0; i < list.arr.size(); ++i) {
        const json::Value& e = list.arr[i];
        const std::string at = "bounding[" + std::to_string(i) + "]";
        Bounding b;
        b.type = str_of(need(e, "type"), at + ".type");
        b.index = ints_of(need(e, "index"), at + ".index");
        if (!all_in(b.index, c.n_output_vars)) bad(at + ".index names an output variable out of range");
        const bool ranged = b.type == "hardtanh" || b.type == "fraction";
        if (b.type != "relu" && !ranged) bad(at + ".type = '" + b.type + "' is not supported (relu, hardtanh, fraction)");
        if (ranged) {
            b.min = float(need(e, "min").as_num((at + ".min").c_str()));
            b.max = float(need(e, "max").as_num((at + ".max").c_str()));
        }
        if (b.type == "fraction") {
            b.total_index = ints_of(need(e, "total_index"), at + ".total_index");
            if (!all_in(b.total_index, c.n_output_vars)) bad(at + ".total_index names an output variable out of range");
            if (b.total_index.size() != 1 && b.total_index.size() != b.index.size())
                bad(at + ".total_index must hold one index or one per entry of index");
        }
        c.bounding.push_back(std::move(b));
    }
}

// blocks: enc.block, proc.0 .. proc.{n-1}, dec.block, each of the kind its position implies
void read_blocks(const json::Value& root, Config& c) {
    const json::Value& blocks = need(root, "blocks");
    const int n = c.num_processor_layers;
    if (int(blocks.size()) != n + 2) bad("blocks must hold enc.block, " + std::to_string(n) + " processor blocks and dec.block");
    for (int i = -1; i <= n; ++i) {
        const bool mapper = i < 0 || i == n;
        const std::string name = i < 0 ? "enc.block" : i == n ? "dec.block" : "proc." + std::to_string(i);
        if (!blocks.has(name)) bad("blocks." + name + " is missing");
        const std::string& kind = str_of(need(blocks.at(name), "kind"), "blocks." + name + ".kind");
        const char* expect = mapper ? "graph_transformer_mapper_block" : "graph_transformer_processor_block";
        if (kind != expect) bad("blocks." + name + ".kind = '" + kind + "' is not supported (" + expect + ")");
        c.block_names.push_back(name);
    }
}

// forcings (optional, rollout): names and model-input indices of the dynamic and constant inputs
void read_forcings(const json::Value& root, Config& c) {
    if (const json::Value* f = find(root, "forcings")) {
        c.has_forcings = true;
        const auto dyn = strs_of(need(*f, "dynamic"), "forcings.dynamic");
        const auto con = strs_of(need(*f, "constant"), "forcings.constant");
        c.forcing_dynamic_index = ints_of(need(*f, "dynamic_input_index"), "forcings.dynamic_input_index");
        c.forcing_constant_index = ints_of(need(*f, "constant_input_index"), "forcings.constant_input_index");
        auto check = [&](const std::vector<std::string>& names, const std::vector<int>& idx, const char* what) {
            if (names.size() != idx.size() || !all_in(idx, c.n_input_vars))
                bad(std::string("forcings.") + what + ": one input index in range per name");
            for (size_t i = 0; i < names.size(); ++i)
                if (c.var_input[size_t(idx[i])] != names[i])
                    bad(std::string("forcings.") + what + ": input " + std::to_string(idx[i]) + " is '" +
                        c.var_input[size_t(idx[i])] + "', not '" + names[i] + "'");
        };
        check(dyn, c.forcing_dynamic_index, "dynamic");
        check(con, c.forcing_constant_index, "constant");
        if (const json::Value* t = find(*f, "timestep_hours")) c.timestep_hours = int(int_of(*t, "forcings.timestep_hours"));
    }
    if (!c.timestep_hours)
        if (const json::Value* t = find(root, "timestep_hours")) c.timestep_hours = int(int_of(*t, "timestep_hours"));
}

}  // namespace

bool Config::is_absent(const std::string& name) const {
    return std::find(absent.begin(), absent.end(), name) != absent.end();
}

Config parse_config(const std::string& text) {
    const json::Value root = json::parse(text);
    Config c;
    c.json_text = text;
    read_scalars(root, c);
    if (c.format_version != 3)
        bad("format_version " + std::to_string(c.format_version) + " is not supported (format 3 only)");
    read_choices(root, c);
    read_lists(root, c);
    if (c.residual_step < 0) c.residual_step += c.n_input_steps;  // negative: counted from the last step
    for (const Rule& r : rules())
        if (!r.holds(c)) bad(std::string("violates: ") + r.what);
    read_bounding(root, c);
    read_blocks(root, c);
    read_forcings(root, c);
    return c;
}

}  // namespace vb
