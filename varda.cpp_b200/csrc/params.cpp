#include "params.h"

#include <map>

namespace vb {

std::vector<TensorSpec> model_schema(const Config& c) {
    const int64_t C = c.num_channels, M = c.mlp_hidden, G = c.n_data_nodes, H = c.n_hidden_nodes;
    const int64_t A = c.node_attr_dim, Ae = c.edge_attr_dim, F = c.src_features(), Vd = c.dec_out_features();
    std::vector<TensorSpec> s = {
        {"norm.mul", DType::F32, {c.n_data_vars}},
        {"norm.add", DType::F32, {c.n_data_vars}},
        {"nodes.data.attr", DType::F32, {G, A}},
        {"nodes.hidden.attr", DType::F32, {H, A}},
    };
    for (const char* g : {"enc", "proc", "dec"}) {
        s.push_back({std::string("graph.") + g + ".edge_index", DType::I64, {2, -1}});
        s.push_back({std::string("graph.") + g + ".edge_attr", DType::F32, {-1, Ae}});
    }
    auto linear = [&](const std::string& n, int64_t out, int64_t in) {
        s.push_back({n + ".weight", DType::F32, {out, in}});
        if (!c.is_absent(n + ".bias")) s.push_back({n + ".bias", DType::F32, {out}});
    };
    auto norm = [&](const std::string& n) {
        s.push_back({n + ".weight", DType::F32, {C}});
        if (!c.is_absent(n + ".bias")) s.push_back({n + ".bias", DType::F32, {C}});
    };
    linear("enc.emb_src", C, F);
    linear("enc.emb_dst", C, A);
    linear("dec.emb_dst", C, F);
    norm("dec.out_norm");
    linear("dec.out_proj", Vd, C);
    for (const std::string& b : c.block_names) {
        const bool mapper = b == "enc.block" || b == "dec.block";
        for (const char* l : {"q", "k", "v", "self", "proj"}) linear(b + "." + l, C, C);
        linear(b + ".mlp1", M, C);
        linear(b + ".mlp2", C, M);
        linear(b + ".edge", C, Ae);
        if (mapper) norm(b + ".ln_src");
        norm(b + ".ln_dst");
        norm(b + ".ln_mlp");
    }
    return s;
}

void validate_model_file(const SafeTensorsFile& f, const Config& c) {
    const std::vector<TensorSpec> schema = model_schema(c);
    std::map<std::string, const TensorSpec*> want;
    for (const TensorSpec& t : schema) want[t.name] = &t;
    auto bad = [&](const std::string& m) { fail(kFormat, f.path() + ": " + m); };
    for (const TensorSpec& t : schema) {
        if (!f.has(t.name)) bad("the model has no tensor '" + t.name + "'");
        const TensorView& v = f.peek(t.name);
        const bool index = t.dtype == DType::I64;  // edge lists: I64 (the format) or I32
        if (!(v.dtype == t.dtype || (index && v.dtype == DType::I32)))
            bad("tensor '" + t.name + "' is " + dtype_name(v.dtype) + ", the format has " + dtype_name(t.dtype));
        bool ok = v.shape.size() == t.shape.size();
        for (size_t i = 0; ok && i < t.shape.size(); ++i) ok = t.shape[i] < 0 || t.shape[i] == v.shape[i];
        if (!ok) {
            std::string w;
            for (int64_t d : t.shape) w += (w.empty() ? "" : ", ") + (d < 0 ? std::string("E") : std::to_string(d));
            bad("tensor '" + t.name + "' has shape " + v.shape_str() + ", the config implies [" + w + "]");
        }
    }
    std::vector<std::string> extra;
    for (const std::string& n : f.names())
        if (!want.count(n) && n != "grid.latitudes" && n != "grid.longitudes") extra.push_back(n);
    if (f.has("grid.latitudes") != f.has("grid.longitudes"))
        bad("grid.latitudes and grid.longitudes come as a pair");
    if (!extra.empty()) {
        std::string list;
        for (size_t i = 0; i < extra.size() && i < 20; ++i) list += (i ? ", " : "") + extra[i];
        bad(std::to_string(extra.size()) + " tensor(s) that a format v3 model with this config does not have: " + list);
    }
}

}  // namespace vb
