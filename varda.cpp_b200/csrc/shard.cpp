#include "shard.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <numeric>

#include "common.h"

namespace vb {

namespace {

// Rank owning index i under contiguous ranges `split` ([world + 1], ascending).
inline int owner_of(const std::vector<int64_t>& split, int64_t i) {
    return int(std::upper_bound(split.begin(), split.end(), i) - split.begin()) - 1;
}

// Contiguous ranges of equal cumulative weight.
std::vector<int64_t> balanced_split(const std::vector<double>& w, int world) {
    const int64_t n = int64_t(w.size());
    std::vector<int64_t> split(size_t(world + 1), n);
    split[0] = 0;
    double total = 0;
    for (double x : w) total += x;
    double acc = 0;
    int r = 1;
    for (int64_t i = 0; i < n && r < world; ++i) {
        acc += w[size_t(i)];
        while (r < world && acc >= total * r / world) split[size_t(r++)] = i + 1;
    }
    for (int k = 1; k <= world; ++k) split[size_t(k)] = std::max(split[size_t(k)], split[size_t(k - 1)]);
    split[size_t(world)] = n;
    return split;
}

// Halos of graph g whose destination rows are owned by `dst_split` and sources by `src_split`.
HaloPlan halos(const CsrGraph& g, const std::vector<int64_t>& dst_split, const std::vector<int64_t>& src_split,
               int world, int rank) {
    HaloPlan h;
    h.recv_count.assign(size_t(world), 0);
    h.send.assign(size_t(world), {});
    for (int p = 0; p < world; ++p) {
        std::vector<int32_t> need;
        const int64_t lo = dst_split[size_t(p)], hi = dst_split[size_t(p + 1)];
        const int64_t slo = src_split[size_t(p)], shi = src_split[size_t(p + 1)];
        for (int64_t e = g.row_ptr[size_t(lo)]; e < g.row_ptr[size_t(hi)]; ++e) {
            const int32_t s = g.src[size_t(e)];
            if (s < slo || s >= shi) need.push_back(s);
        }
        std::sort(need.begin(), need.end());
        need.erase(std::unique(need.begin(), need.end()), need.end());
        if (p == rank) {
            h.halo = need;
            for (int32_t s : need) ++h.recv_count[size_t(owner_of(src_split, s))];
        } else {
            const int64_t mlo = src_split[size_t(rank)], mhi = src_split[size_t(rank + 1)];
            auto a = std::lower_bound(need.begin(), need.end(), int32_t(mlo));
            auto b = std::lower_bound(need.begin(), need.end(), int32_t(mhi));
            h.send[size_t(p)].assign(a, b);
        }
    }
    return h;
}

// Rows [lo, hi) of g with sources remapped to local ids: own sources [slo, shi) -> s - slo, halo
// sources -> (shi - slo) + position in `halo`. Edge order within a row is kept.
CsrGraph local_graph(const CsrGraph& g, int64_t lo, int64_t hi, int64_t slo, int64_t shi,
                     const std::vector<int32_t>& halo) {
    CsrGraph l;
    l.n_dst = hi - lo;
    l.n_src = (shi - slo) + int64_t(halo.size());
    l.attr_dim = g.attr_dim;
    const int64_t e0 = g.row_ptr[size_t(lo)], e1 = g.row_ptr[size_t(hi)];
    l.n_edges = e1 - e0;
    l.row_ptr.resize(size_t(l.n_dst + 1));
    for (int64_t d = 0; d <= l.n_dst; ++d) l.row_ptr[size_t(d)] = int32_t(g.row_ptr[size_t(lo + d)] - e0);
    l.src.resize(size_t(l.n_edges));
    l.edge_id.assign(g.edge_id.begin() + e0, g.edge_id.begin() + e1);
    l.attr.assign(g.attr.begin() + e0 * g.attr_dim, g.attr.begin() + e1 * g.attr_dim);
    for (int64_t e = e0; e < e1; ++e) {
        const int32_t s = g.src[size_t(e)];
        int64_t ls;
        if (s >= slo && s < shi) {
            ls = s - slo;
        } else {
            auto it = std::lower_bound(halo.begin(), halo.end(), s);
            if (it == halo.end() || *it != s) fail(kInternal, "shard plan: a source is missing from the halo");
            ls = (shi - slo) + (it - halo.begin());
        }
        l.src[size_t(e - e0)] = int32_t(ls);
    }
    return l;
}

}  // namespace

// The encoder's own hidden split is the default (VB_SHARD_ENC=0 turns it off): on C1 at 2 B200 it took
// the step from 93.4 to 90.3 ms and rank 0's halo-exchange wait from 11.0 to 1.8 ms.
bool enc_split_requested() {
    const char* e = std::getenv("VB_SHARD_ENC");
    return !(e && *e && std::atoi(e) == 0);
}

ShardPlan make_plan(const Config& c, const CsrGraph& enc, const CsrGraph& proc, const CsrGraph& dec, int world,
                    int rank, bool enc_split) {
    if (world < 1 || rank < 0 || rank >= world) fail(kInvalidArgument, "shard plan: bad rank/world");
    ShardPlan p;
    p.world = world, p.rank = rank;
    const int64_t G = c.n_data_nodes, H = c.n_hidden_nodes;
    if (world == 1) {
        p.h_split = {0, H};
        p.g_split = {0, G};
        p.e_split = p.h_split;
    } else {
        if (H < world) fail(kUnsupported, "shard plan: fewer hidden nodes than GPUs");
        if (G < world) fail(kUnsupported, "shard plan: fewer data nodes than GPUs");
        // Cost model (seconds-equivalents): GEMM FLOPs at ~1.2 PFLOP/s, edge gathers at ~5 TB/s. The step
        // is a chain of phases with a halo exchange between them (encoder, 16 processor blocks,
        // decoder), so each phase is balanced on its own: hidden rows on the processor work, data rows
        // on the encoder-source and decoder work.
        const double C = c.num_channels, M = c.mlp_hidden, F = double(align_up(size_t(c.src_features()), 8));
        const double P = c.num_processor_layers, Vd = c.dec_out_features();
        const double kF = 1.0 / 1.2e15, kB = 1.0 / 5e12, row_bytes = 2.0 * C * 2.0;
        const double flop_h = 2 * C * 2 * C + 2 * C * C + 4 * C * M + P * (2 * C * 4 * C + 2 * C * C + 4 * C * M) +
                              2 * C * 2 * C;
        const double flop_g = 2 * F * C + 2 * C * 2 * C + 2 * F * C + 2 * C * 2 * C + 2 * C * C + 4 * C * M + 2 * C * Vd;
        std::vector<double> wh(static_cast<size_t>(H)), wg(static_cast<size_t>(G));
        // the encoder's gathers (one phase, concentrated on the dense region's hidden rows) are left
        // out of the hidden weights: the 16 processor phases dominate and need equal shares
        for (int64_t h = 0; h < H; ++h)
            wh[size_t(h)] = flop_h * kF +
                            P * (proc.row_ptr[size_t(h + 1)] - proc.row_ptr[size_t(h)]) * row_bytes * 0.5 * kB;
        for (int64_t g = 0; g < G; ++g)
            wg[size_t(g)] = flop_g * kF + (dec.row_ptr[size_t(g + 1)] - dec.row_ptr[size_t(g)]) * row_bytes * kB;
        p.h_split = balanced_split(wh, world);
        // hidden ranges start on the tensor-core attention's tile grid (every kTcAlignRows rows) when the
        // graph is large enough for it, so each rank's processor tiles are the single GPU's tiles and
        // the results stay bitwise independent of the GPU count
        if (H >= 2 * kTcAlignRows * world) {
            for (int k = 1; k < world; ++k) {
                const int64_t r = (p.h_split[size_t(k)] + kTcAlignRows / 2) / kTcAlignRows * kTcAlignRows;
                p.h_split[size_t(k)] = std::min(H, std::max(p.h_split[size_t(k - 1)] + kTcAlignRows, r));
            }
        }
        p.g_split = balanced_split(wg, world);
        p.e_split = p.h_split;
        if (enc_split) {
            // encoder phase alone: destination-side GEMMs per hidden row; per encoder edge its K|V read
            // and its share of the source side (the data rows a range reads are recomputed or owned
            // there, about E_enc / G edges per data row)
            const double A = c.node_attr_dim;
            const double flop_he = 2 * A * C + 2 * C * 2 * C + 2 * C * C + 4 * C * M;
            const double flop_gs = 2 * F * C + 2 * C * 2 * C;
            const double per_edge = row_bytes * kB + flop_gs * kF * double(G) / double(std::max<int64_t>(enc.n_edges, 1));
            std::vector<double> we(static_cast<size_t>(H));
            for (int64_t h = 0; h < H; ++h)
                we[size_t(h)] = flop_he * kF + (enc.row_ptr[size_t(h + 1)] - enc.row_ptr[size_t(h)]) * per_edge;
            std::vector<int64_t> es = balanced_split(we, world);
            bool nonempty = true;  // an empty encoder range keeps the processor's ranges
            for (int k = 0; k < world; ++k) nonempty = nonempty && es[size_t(k + 1)] > es[size_t(k)];
            if (nonempty) p.e_split = es;
        }
    }
    p.h_lo = p.h_split[size_t(rank)], p.h_hi = p.h_split[size_t(rank + 1)];
    p.g_lo = p.g_split[size_t(rank)], p.g_hi = p.g_split[size_t(rank + 1)];
    p.e_lo = p.e_split[size_t(rank)], p.e_hi = p.e_split[size_t(rank + 1)];
    for (int q = 0; q < world; ++q) {
        p.enc_move.send_lo.push_back(std::max(p.e_lo, p.h_split[size_t(q)]));
        p.enc_move.send_hi.push_back(std::min(p.e_hi, p.h_split[size_t(q + 1)]));
        p.enc_move.recv_lo.push_back(std::max(p.h_lo, p.e_split[size_t(q)]));
        p.enc_move.recv_hi.push_back(std::min(p.h_hi, p.e_split[size_t(q + 1)]));
    }

    p.proc = halos(proc, p.h_split, p.h_split, world, rank);
    p.dec = halos(dec, p.g_split, p.h_split, world, rank);
    // encoder: remote data sources of own encoder rows (their inputs come from their owners, their source
    // side is recomputed here)
    p.enc_x = halos(enc, p.e_split, p.g_split, world, rank);
    p.enc_halo = p.enc_x.halo;

    p.enc = local_graph(enc, p.e_lo, p.e_hi, p.g_lo, p.g_hi, p.enc_halo);
    p.proc_g = local_graph(proc, p.h_lo, p.h_hi, p.h_lo, p.h_hi, p.proc.halo);
    p.dec_g = local_graph(dec, p.g_lo, p.g_hi, p.h_lo, p.h_hi, p.dec.halo);
    return p;
}

namespace {
template <class V> void put_list(std::string& o, const V& v) {
    o += "[";
    for (size_t i = 0; i < v.size(); ++i) {
        if (i) o += ",";
        o += std::to_string(v[i]);
    }
    o += "]";
}
void put_halo(std::string& o, const HaloPlan& h) {
    o += "{\"halo\":";
    put_list(o, h.halo);
    o += ",\"recv_count\":";
    put_list(o, h.recv_count);
    o += ",\"send\":[";
    for (size_t i = 0; i < h.send.size(); ++i) {
        if (i) o += ",";
        put_list(o, h.send[i]);
    }
    o += "]}";
}
void put_graph(std::string& o, const CsrGraph& g) {
    o += "{\"n_src\":" + std::to_string(g.n_src) + ",\"row_ptr\":";
    put_list(o, g.row_ptr);
    o += ",\"src\":";
    put_list(o, g.src);
    o += ",\"edge_id\":";
    put_list(o, g.edge_id);
    o += "}";
}
}  // namespace

std::string plan_json(const ShardPlan& p, bool with_graphs) {
    std::string o = "{\"world\":" + std::to_string(p.world) + ",\"rank\":" + std::to_string(p.rank) + ",\"h_split\":";
    put_list(o, p.h_split);
    o += ",\"g_split\":";
    put_list(o, p.g_split);
    o += ",\"e_split\":";
    put_list(o, p.e_split);
    o += ",\"enc_move\":{\"send_lo\":";
    put_list(o, p.enc_move.send_lo);
    o += ",\"send_hi\":";
    put_list(o, p.enc_move.send_hi);
    o += ",\"recv_lo\":";
    put_list(o, p.enc_move.recv_lo);
    o += ",\"recv_hi\":";
    put_list(o, p.enc_move.recv_hi);
    o += "}";
    o += ",\"proc\":";
    put_halo(o, p.proc);
    o += ",\"dec\":";
    put_halo(o, p.dec);
    o += ",\"enc_halo\":";
    put_list(o, p.enc_halo);
    if (with_graphs) {
        o += ",\"enc\":";
        put_graph(o, p.enc);
        o += ",\"proc_g\":";
        put_graph(o, p.proc_g);
        o += ",\"dec_g\":";
        put_graph(o, p.dec_g);
    }
    return o + "}";
}

}  // namespace vb
