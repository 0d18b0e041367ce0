#include "graph.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <array>
#include <cstring>
#include <limits>
#include <string>
#include <thread>
#include <vector>

#include "common.h"

namespace vb {

int32_t CsrGraph::max_degree() const {
    int32_t m = 0;
    for (int64_t d = 0; d < n_dst; ++d) m = std::max(m, row_ptr[d + 1] - row_ptr[d]);
    return m;
}

namespace {

// Threads for the host-side graph passes: a few for large graphs, one below kParallelEdges edges.
constexpr int64_t kParallelEdges = 1 << 20;
int graph_threads(int64_t E) {
    if (E < kParallelEdges) return 1;
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    return int(std::min<int64_t>(std::min<unsigned>(hw, 16u), E / (kParallelEdges / 2)));
}
template <class F> void parallel_chunks(int nt, int64_t n, F f) {  // f(t, begin, end) on nt threads
    if (nt <= 1) return f(0, int64_t(0), n);
    std::vector<std::thread> ts;
    for (int t = 0; t < nt; ++t) ts.emplace_back(f, t, n * t / nt, n * (t + 1) / nt);
    for (auto& th : ts) th.join();
}

// Stable counting sort by destination on nt threads: thread t counts the destinations of its
// contiguous edge range, every destination's slots are handed out to the threads in range order, and
// each thread scatters its range in order, so the result is the one-thread order exactly.
template <class I>
CsrGraph build(const I* ei, int64_t E, const float* ea, int A, int64_t n_src, int64_t n_dst, const std::string& name) {
    constexpr int64_t kMax = std::numeric_limits<int32_t>::max();
    if (E >= kMax || n_src >= kMax || n_dst >= kMax) fail(kFormat, name + ": graph too large for int32 indices");
    CsrGraph g;
    g.n_src = n_src;
    g.n_dst = n_dst;
    g.n_edges = E;
    g.attr_dim = A;
    const int nt = graph_threads(E);
    std::vector<std::vector<int32_t>> cnt(size_t(nt), std::vector<int32_t>(size_t(n_dst), 0));
    std::vector<int64_t> bad(size_t(nt), -1);  // first out-of-range edge of each thread's range
    parallel_chunks(nt, E, [&](int t, int64_t b, int64_t e) {
        int32_t* c = cnt[size_t(t)].data();
        for (int64_t i = b; i < e; ++i) {
            const int64_t s = int64_t(ei[i]), d = int64_t(ei[E + i]);
            if (s < 0 || s >= n_src || d < 0 || d >= n_dst) {
                bad[size_t(t)] = i;
                return;
            }
            ++c[d];
        }
    });
    for (int t = 0; t < nt; ++t)
        if (bad[size_t(t)] >= 0) fail(kFormat, name + ": edge " + std::to_string(bad[size_t(t)]) + " out of range");
    g.row_ptr.assign(size_t(n_dst + 1), 0);
    for (int64_t d = 0; d < n_dst; ++d) {  // row_ptr, and cnt[t][d] becomes thread t's first slot of d
        int32_t off = g.row_ptr[size_t(d)];
        for (int t = 0; t < nt; ++t) {
            const int32_t c = cnt[size_t(t)][size_t(d)];
            cnt[size_t(t)][size_t(d)] = off;
            off += c;
        }
        g.row_ptr[size_t(d + 1)] = off;
    }
    g.src.resize(size_t(E));
    g.edge_id.resize(size_t(E));
    g.attr.resize(size_t(E) * size_t(A));
    parallel_chunks(nt, E, [&](int t, int64_t b, int64_t e) {
        int32_t* next = cnt[size_t(t)].data();
        for (int64_t i = b; i < e; ++i) {
            const int32_t slot = next[ei[E + i]]++;
            g.src[size_t(slot)] = int32_t(ei[i]);
            g.edge_id[size_t(slot)] = int32_t(i);
            std::memcpy(&g.attr[size_t(slot) * size_t(A)], ea + i * A, sizeof(float) * size_t(A));
        }
    });
    return g;
}
}  // namespace

CsrGraph build_csr_by_dst(const TensorView& ei, const TensorView& ea, int64_t n_src, int64_t n_dst) {
    if (ei.shape.size() != 2 || ei.shape[0] != 2)
        fail(kFormat, ei.name + ": expected shape [2, E], got " + ei.shape_str());
    const int64_t E = ei.shape[1];
    if (ea.dtype != DType::F32 || ea.shape.size() != 2 || ea.shape[0] != E)
        fail(kFormat, ea.name + ": expected F32 [E, A] with E = " + std::to_string(E));
    const int A = int(ea.shape[1]);
    if (ei.dtype == DType::I64) return build(ei.as<int64_t>(), E, ea.as<float>(), A, n_src, n_dst, ei.name);
    if (ei.dtype == DType::I32) return build(ei.as<int32_t>(), E, ea.as<float>(), A, n_src, n_dst, ei.name);
    fail(kFormat, ei.name + ": edge_index must be I64 or I32");
}

CsrGraph build_csr_by_dst(const int64_t* ei, int64_t E, const float* ea, int A, int64_t n_src, int64_t n_dst) {
    return build(ei, E, ea, A, n_src, n_dst, "edge_index");
}

std::vector<EdgeRec> pack_edges(const CsrGraph& g, bool round_fp16) {
    if (g.attr_dim > 3) fail(kUnsupported, "edge_attr_dim must be 1..3 (16-byte edge records)");
    std::vector<EdgeRec> out(size_t(g.n_edges));
    parallel_chunks(graph_threads(g.n_edges), g.n_edges, [&](int, int64_t b, int64_t end) {
        for (int64_t e = b; e < end; ++e) {
            float a[3] = {0.f, 0.f, 0.f};
            for (int k = 0; k < g.attr_dim; ++k) {
                const float v = g.attr[size_t(e) * size_t(g.attr_dim) + size_t(k)];
                a[k] = round_fp16 ? __half2float(__float2half_rn(v)) : v;
            }
            out[size_t(e)] = {a[0], a[1], a[2], g.src[size_t(e)]};
        }
    });
    return out;
}

TilePlan make_tiles(const CsrGraph& g, int max_src, int max_rows, int max_edges, int64_t chunk_rows, bool round_fp16,
                    int max_row_edges, bool sort_by_slot) {
    TilePlan t;
    t.edges = pack_edges(g, round_fp16);
    std::vector<int32_t> slot(size_t(std::max<int64_t>(g.n_src, 1)), -1);  // source -> slot in the open tile
    std::vector<int32_t> open;                                             // distinct sources of the open tile
    int32_t row0 = -1;
    auto close = [&](int64_t end_row) {
        if (row0 < 0) return;
        std::vector<int32_t> sorted = open;
        std::sort(sorted.begin(), sorted.end());
        for (size_t i = 0; i < sorted.size(); ++i) slot[size_t(sorted[i])] = int32_t(i);
        for (int64_t e = g.row_ptr[size_t(row0)]; e < g.row_ptr[size_t(end_row)]; ++e)
            t.edges[size_t(e)].src = slot[size_t(g.src[size_t(e)])];
        if (sort_by_slot)
            for (int64_t d = row0; d < end_row; ++d)
                std::stable_sort(t.edges.begin() + g.row_ptr[size_t(d)], t.edges.begin() + g.row_ptr[size_t(d + 1)],
                                 [](const EdgeRec& x, const EdgeRec& y) { return x.src < y.src; });
        t.row0.push_back(row0);
        t.nrows.push_back(int32_t(end_row - row0));
        t.src0.push_back(int32_t(t.srcs.size()));
        t.nsrc.push_back(int32_t(sorted.size()));
        t.max_nsrc = std::max(t.max_nsrc, int(sorted.size()));
        t.srcs.insert(t.srcs.end(), sorted.begin(), sorted.end());
        for (int32_t s : open) slot[size_t(s)] = -1;
        open.clear();
        row0 = -1;
    };
    std::vector<int32_t> fresh;
    for (int64_t d = 0; d < g.n_dst; ++d) {
        const int32_t b = g.row_ptr[size_t(d)], e = g.row_ptr[size_t(d + 1)];
        if (chunk_rows > 0 && d % chunk_rows == 0) close(d);
        // distinct sources of row d not yet in the open tile (slot -2 marks "seen in this row")
        fresh.clear();
        for (int32_t i = b; i < e; ++i) {
            const int32_t s = g.src[size_t(i)];
            if (slot[size_t(s)] == -1) slot[size_t(s)] = -2, fresh.push_back(s);
        }
        int own = 0;  // distinct sources of the row alone
        {
            std::vector<int32_t> u(g.src.begin() + b, g.src.begin() + e);
            std::sort(u.begin(), u.end());
            own = int(std::unique(u.begin(), u.end()) - u.begin());
        }
        for (int32_t s : fresh) slot[size_t(s)] = -1;
        if (own > max_src || e - b > max_edges || (max_row_edges > 0 && e - b > max_row_edges)) {  // heavy row
            close(d);
            t.heavy.push_back(int32_t(d));
            continue;
        }
        const bool fits = row0 >= 0 && int(open.size() + fresh.size()) <= max_src && d - row0 < max_rows &&
                          e - g.row_ptr[size_t(row0)] <= max_edges;
        if (!fits) {
            close(d);
            row0 = int32_t(d);
            fresh.clear();
            for (int32_t i = b; i < e; ++i) {
                const int32_t s = g.src[size_t(i)];
                if (slot[size_t(s)] == -1) slot[size_t(s)] = -2, fresh.push_back(s);
            }
        }
        for (int32_t s : fresh) slot[size_t(s)] = -3, open.push_back(s);  // -3: in the open tile
    }
    close(g.n_dst);
    return t;
}

TcPlan make_tc_tiles(const CsrGraph& g, int64_t align_rows) {
    if (g.attr_dim > 3) fail(kUnsupported, "edge_attr_dim must be 1..3");
    TcPlan t;
    std::vector<int32_t> slot(size_t(std::max<int64_t>(g.n_src, 1)), -1);  // source -> slot in the open tile
    std::vector<int32_t> open;                                             // the open tile's sources, by slot
    int64_t row0 = -1;
    auto half_bits = [](float v) {
        const __half h = __float2half_rn(v);
        uint16_t b;
        std::memcpy(&b, &h, 2);
        return b;
    };
    auto close = [&](int64_t end_row) {
        if (row0 < 0) return;
        const int64_t e0 = g.row_ptr[size_t(row0)], e1 = g.row_ptr[size_t(end_row)];
        const int nrows = int(end_row - row0), ne = int(e1 - e0);
        const int nb = (nrows + 15) / 16;
        // slot order: by the first 16-row block that reads the source, then by the last one, then by first
        // appearance (stable), so each block's private sources come first in its range and the sources it
        // shares with the next blocks sit next to theirs: a block's edges fall into fewer 8-slot column
        // blocks (4.4 per block on the C2 graph against 5.2 in plain first-appearance order). The order
        // depends only on the tile's rows and edges, not on how the graph's nodes are numbered.
        {
            std::vector<int> fb(open.size(), nb), lb(open.size(), -1);
            for (int i = 0; i < nrows; ++i)
                for (int64_t x = g.row_ptr[size_t(row0 + i)]; x < g.row_ptr[size_t(row0 + i + 1)]; ++x) {
                    const size_t k = size_t(slot[size_t(g.src[size_t(x)])]);
                    fb[k] = std::min(fb[k], i / 16), lb[k] = std::max(lb[k], i / 16);
                }
            std::vector<int32_t> ord(open.size());
            for (size_t k = 0; k < ord.size(); ++k) ord[k] = int32_t(k);
            std::stable_sort(ord.begin(), ord.end(), [&](int32_t x, int32_t y) {
                return fb[size_t(x)] != fb[size_t(y)] ? fb[size_t(x)] < fb[size_t(y)] : lb[size_t(x)] < lb[size_t(y)];
            });
            std::vector<int32_t> sorted(open.size());
            for (size_t k = 0; k < ord.size(); ++k) sorted[k] = open[size_t(ord[k])];
            open.swap(sorted);
            for (size_t k = 0; k < open.size(); ++k) slot[size_t(open[k])] = int32_t(k);
        }
        // per 16-row block: the column blocks holding edges, and each (row, slot)'s edge index in its row
        std::vector<std::vector<int>> cols(static_cast<size_t>(nb));
        std::vector<std::array<uint8_t, 16 * kTcMaxSrc>> at(static_cast<size_t>(nb));
        for (auto& a : at) a.fill(255);
        for (int i = 0; i < nrows; ++i) {
            const int64_t b = g.row_ptr[size_t(row0 + i)], e = g.row_ptr[size_t(row0 + i + 1)];
            for (int64_t x = b; x < e; ++x) {
                const int32_t sl = slot[size_t(g.src[size_t(x)])];
                at[size_t(i / 16)][size_t((i % 16) * kTcMaxSrc + sl)] = uint8_t(x - b);
            }
        }
        int n_chunks = 0;
        std::vector<int> chunk0(static_cast<size_t>(nb));
        for (int bk = 0; bk < nb; ++bk) {
            bool used[kTcMaxSrc / 8] = {};
            for (int r = 0; r < 16; ++r)
                for (int sl = 0; sl < kTcMaxSrc; ++sl)
                    if (at[size_t(bk)][size_t(r * kTcMaxSrc + sl)] != 255) used[sl / 8] = true;
            auto& cl = cols[size_t(bk)];
            for (int j = 0; j < kTcMaxSrc / 8; ++j)
                if (used[j]) cl.push_back(j);
            if (cl.size() % 2) cl.push_back(-1 - cl.back());  // an empty repeat of the last block
            chunk0[size_t(bk)] = n_chunks;
            n_chunks += int(cl.size() / 2);
        }
        TcTile tile{};
        tile.row0 = int32_t(row0), tile.nrows = nrows, tile.nsrc = int32_t(open.size());
        tile.src_off = int32_t(t.srcs.size());
        tile.blob_off = int32_t(t.blob.size()), tile.n_edges = ne;
        tile.attr_off = kTcMaskOff + 32 * n_chunks;
        tile.blob_bytes = tile.attr_off + kTcChunkAttr * n_chunks;
        t.srcs.insert(t.srcs.end(), open.begin(), open.end());
        while (t.srcs.size() % 4) t.srcs.push_back(open.back());
        t.blob.resize(t.blob.size() + size_t(tile.blob_bytes), 0);
        uint8_t* bl = t.blob.data() + tile.blob_off;
        for (int bk = 0; bk < nb; ++bk) {
            uint8_t* hd = bl + kTcBlockOff + 32 * bk;
            const auto& cl = cols[size_t(bk)];
            hd[0] = uint8_t(cl.size() / 2), hd[1] = uint8_t(chunk0[size_t(bk)]);
            for (size_t k = 0; k < cl.size(); ++k) hd[2 + k] = uint8_t(cl[k] >= 0 ? cl[k] : -1 - cl[k]);
            for (size_t c = 0; c < cl.size() / 2; ++c) {
                const int ci = chunk0[size_t(bk)] + int(c);
                uint8_t* mask = bl + kTcMaskOff + 32 * ci;
                uint16_t* attr = reinterpret_cast<uint16_t*>(bl + tile.attr_off + size_t(kTcChunkAttr) * size_t(ci));
                for (int l = 0; l < 32; ++l) {
                    const int r = l / 4, tq = l % 4;
                    for (int e = 0; e < 8; ++e) {
                        const int j = cl[2 * c + size_t(e >> 2)];  // column block (negative: the padding)
                        const int row = r + 8 * ((e >> 1) & 1), sl = 8 * (j >= 0 ? j : 0) + 2 * tq + (e & 1);
                        const int idx = j >= 0 ? at[size_t(bk)][size_t(row * kTcMaxSrc + sl)] : 255;
                        if (idx == 255) continue;
                        mask[l] = uint8_t(mask[l] | (1u << e));
                        const int64_t x = g.row_ptr[size_t(row0 + 16 * bk + row)] + idx;  // the edge
                        for (int k = 0; k < 3; ++k)  // word 3 (e / 2) + k, half e % 2
                            attr[24 * l + 2 * (3 * (e >> 1) + k) + (e & 1)] =
                                half_bits(k < g.attr_dim ? g.attr[size_t(x) * size_t(g.attr_dim) + size_t(k)] : 0.f);
                    }
                }
            }
        }
        t.tiles.push_back(tile);
        for (int32_t s : open) slot[size_t(s)] = -1;
        open.clear();
        row0 = -1;
    };
    std::vector<int32_t> fresh, u;
    for (int64_t d = 0; d < g.n_dst; ++d) {
        if (align_rows > 0 && d % align_rows == 0) close(d);
        const int32_t b = g.row_ptr[size_t(d)], e = g.row_ptr[size_t(d + 1)];
        u.assign(g.src.begin() + b, g.src.begin() + e);
        std::sort(u.begin(), u.end());
        const bool dup = std::adjacent_find(u.begin(), u.end()) != u.end();
        if (dup || e - b > kTcMaxEdges || int64_t(u.size()) > kTcMaxSrc) {
            close(d);
            t.heavy.push_back(int32_t(d));
            continue;
        }
        // the row's sources not yet in the open tile, in edge order (no duplicates within the row)
        fresh.clear();
        for (int32_t i = b; i < e; ++i)
            if (slot[size_t(g.src[size_t(i)])] < 0) fresh.push_back(g.src[size_t(i)]);
        const bool fits = row0 >= 0 && open.size() + fresh.size() <= size_t(kTcMaxSrc) && d - row0 < kTcRows &&
                          e - g.row_ptr[size_t(row0)] <= kTcMaxEdges;
        if (!fits && row0 >= 0 && d - row0 > 16 && (d - row0) % 16) {
            // end the tile at its last whole 16-row block (the kernel's unit of work) and take the rows
            // after it again into the next tile: fewer, fuller blocks (C2: 11,866 blocks against 14,686)
            const int64_t end = row0 + (d - row0) / 16 * 16;
            for (int32_t s : open) slot[size_t(s)] = -1;
            open.clear();
            for (int64_t x = g.row_ptr[size_t(row0)]; x < g.row_ptr[size_t(end)]; ++x)
                if (slot[size_t(g.src[size_t(x)])] < 0)
                    slot[size_t(g.src[size_t(x)])] = int32_t(open.size()), open.push_back(g.src[size_t(x)]);
            close(end);
            d = end - 1;  // the loop goes on at row `end`
            continue;
        }
        if (!fits) {
            close(d);
            row0 = d;
            fresh.assign(g.src.begin() + b, g.src.begin() + e);
        }
        for (int32_t s : fresh) slot[size_t(s)] = int32_t(open.size()), open.push_back(s);
    }
    close(g.n_dst);
    return t;
}

}  // namespace vb
