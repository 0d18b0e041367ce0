// The C ABI (include/varda_b200.h) over the C++ engine: exceptions become status codes plus a
// thread-local message.
#include "../../include/varda_b200.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>

#include "comm.h"
#include "common.h"
#include "config.h"
#include "engine.h"
#include "safetensors.h"
#include "gemm_tc.cuh"
#include "graph.h"
#include "kernels.cuh"
#include "shard.h"

struct vb_model {
    std::unique_ptr<vb::Model> m;
};

namespace {

thread_local std::string g_last_error;

template <class F> int guard(F&& f) {
    try {
        f();
        g_last_error.clear();
        return VB_OK;
    } catch (const vb::Error& e) {
        g_last_error = e.what();
        return e.cls;
    } catch (const std::bad_alloc&) {
        g_last_error = "out of host memory";
        return VB_ERR_INTERNAL;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return VB_ERR_INTERNAL;
    } catch (...) {
        g_last_error = "unknown error";
        return VB_ERR_INTERNAL;
    }
}

cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

vb::Options to_opts(const vb_options* o) {
    vb::Options r;
    if (o) {
        if (o->precision != VB_PRECISION_FP32 && o->precision != VB_PRECISION_FP16)
            vb::fail(vb::kInvalidArgument, "precision must be VB_PRECISION_FP32 or VB_PRECISION_FP16");
        r.precision = o->precision;
        r.cuda_device = o->cuda_device;
        r.cuda_graph = o->cuda_graph != 0;
    }
    return r;
}

void need(const void* p, const char* what) {
    if (!p) vb::fail(vb::kInvalidArgument, std::string(what) + " is NULL");
}

// The kernels' device-side timeout flags (read and cleared; synchronises the device).
void device_errors() {
    if (vb::tc::take_error()) vb::fail(vb::kTimeout, "a device-side wait timed out in the tensor-core GEMM");
    if (vb::k::take_attention_error()) vb::fail(vb::kTimeout, "a device-side wait timed out in the attention");
}

}  // namespace

extern "C" {

const char* vb_last_error(void) { return g_last_error.c_str(); }

int vb_load(const char* path, const vb_options* opts, vb_model** out) {
    return guard([&] {
        need(path, "path");
        need(out, "out");
        *out = nullptr;
        auto m = std::make_unique<vb_model>();
        m->m = vb::load_model(path, to_opts(opts));
        *out = m.release();
    });
}

int vb_load_sharded(const char* path, const vb_options* opts, int rank, int world, const void* nccl_id,
                    vb_model** out) {
    return guard([&] {
        need(path, "path");
        need(out, "out");
        *out = nullptr;
        if (world < 1 || rank < 0 || rank >= world) vb::fail(vb::kInvalidArgument, "bad rank / world");
        vb::Options o = to_opts(opts);
        o.rank = rank, o.world = world, o.nccl_id = nccl_id;
        if (world > 1) need(nccl_id, "nccl_id");
        auto m = std::make_unique<vb_model>();
        m->m = vb::load_model(path, o);
        *out = m.release();
    });
}

int vb_nccl_unique_id(void* out128) {
    return guard([&] {
        need(out128, "out");
        vb::nccl_unique_id(out128);
    });
}

void vb_free(vb_model* m) { delete m; }

int vb_predict_step(vb_model* m, const float* x, float* y, vb_hook_fn hook, void* user) {
    return guard([&] {
        need(m, "model"), need(x, "x"), need(y, "y");
        m->m->predict_step(x, y, hook, user);
        device_errors();
    });
}

int vb_rollout(vb_model* m, const float* x0, int n_steps, const float* forcings, float* y, int constants_oldest,
               vb_step_fn on_step, void* user, float* step_ms) {
    return guard([&] {
        need(m, "model"), need(x0, "x0");
        m->m->rollout(x0, n_steps, forcings, y, constants_oldest != 0, on_step, user, step_ms);
        device_errors();
    });
}

int vb_sizes(const vb_model* m, int64_t out8[8]) {
    return guard([&] {
        need(m, "model"), need(out8, "out");
        m->m->sizes(out8);
    });
}

int vb_data_range(const vb_model* m, int64_t* lo, int64_t* hi) {
    return guard([&] {
        need(m, "model"), need(lo, "lo"), need(hi, "hi");
        m->m->data_range(lo, hi);
    });
}

int vb_hidden_range(const vb_model* m, int64_t* lo, int64_t* hi) {
    return guard([&] {
        need(m, "model"), need(lo, "lo"), need(hi, "hi");
        m->m->hidden_range(lo, hi);
    });
}

int vb_processor_block(vb_model* m, int block, const float* z_in, float* z_out, int repeats, float* device_ms) {
    return guard([&] {
        need(m, "model");
        m->m->processor_block(block, z_in, z_out, repeats, device_ms);
    });
}

int vb_io_numel(const vb_model* m, int64_t* in, int64_t* out) {
    return guard([&] {
        need(m, "model"), need(in, "in"), need(out, "out");
        *in = m->m->input_numel(), *out = m->m->output_numel();
    });
}

int vb_normalise(vb_model* m, const float* x, float* xn, void* stream) {
    return guard([&] {
        need(m, "model"), need(x, "x"), need(xn, "xn");
        m->m->normalise(x, xn, S(stream));
    });
}
int vb_forward_normalised(vb_model* m, const float* xn, float* yn, void* stream) {
    return guard([&] {
        need(m, "model"), need(xn, "xn"), need(yn, "yn");
        m->m->forward_normalised(xn, yn, S(stream));
    });
}
int vb_denormalise(vb_model* m, const float* yn, float* y, void* stream) {
    return guard([&] {
        need(m, "model"), need(yn, "yn"), need(y, "y");
        m->m->denormalise(yn, y, S(stream));
    });
}
int vb_predict_step_device(vb_model* m, const float* x, float* y, void* stream) {
    return guard([&] {
        need(m, "model"), need(x, "x"), need(y, "y");
        m->m->predict_step_device(x, y, S(stream));
    });
}
int vb_prepare(vb_model* m) {
    return guard([&] {
        need(m, "model");
        m->m->prepare();
    });
}
int vb_use_high_priority_stream(vb_model* m) {
    return guard([&] {
        need(m, "model");
        m->m->use_high_priority_stream();
    });
}
float* vb_device_input(vb_model* m) { return m ? m->m->device_input() : nullptr; }
const float* vb_device_output(vb_model* m) { return m ? m->m->device_output() : nullptr; }
void* vb_stream(vb_model* m) { return m ? static_cast<void*>(m->m->stream()) : nullptr; }
int vb_enqueue_predict(vb_model* m) {
    return guard([&] {
        need(m, "model");
        m->m->enqueue_predict();
    });
}
int vb_device(const vb_model* m) { return m ? m->m->device() : -1; }
size_t vb_weight_bytes(const vb_model* m) { return m ? m->m->weight_bytes() : 0; }
size_t vb_activation_bytes(const vb_model* m) { return m ? m->m->activation_bytes() : 0; }
int64_t vb_decoder_chunk_rows(const vb_model* m) { return m ? m->m->decoder_chunk_rows() : 0; }

int vb_check_device(void) {
    return guard([&] { device_errors(); });
}

int64_t vb_shard_plan(const char* path, int world, int rank, char* buf, size_t len) {
    std::string s;
    const int rc = guard([&] {
        need(path, "path");
        vb::SafeTensorsFile f(path);
        const vb::Config c = vb::parse_config(f.metadata("config"));
        const int64_t G = c.n_data_nodes, H = c.n_hidden_nodes;
        auto g = [&](const char* n, int64_t ns, int64_t nd) {
            return vb::build_csr_by_dst(f.peek(std::string("graph.") + n + ".edge_index"),
                                        f.peek(std::string("graph.") + n + ".edge_attr"), ns, nd);
        };
        const vb::CsrGraph enc = g("enc", G, H), proc = g("proc", H, H), dec = g("dec", H, G);
        s = vb::plan_json(vb::make_plan(c, enc, proc, dec, world, rank, vb::enc_split_requested()), true);
    });
    if (rc != VB_OK) return -rc;
    if (buf && len) {
        const size_t n = std::min(len - 1, s.size());
        std::memcpy(buf, s.data(), n);
        buf[n] = 0;
    }
    return int64_t(s.size() + 1);
}

int64_t vb_launch_count(void) { return vb::launch_counter().load(); }

int64_t vb_profile_forward(vb_model* m, char* buf, size_t len) {
    std::string s;
    const int rc = guard([&] {
        need(m, "model");
        s = m->m->profile_forward();
    });
    if (rc != VB_OK) return -rc;
    if (buf && len) {
        const size_t n = std::min(len - 1, s.size());
        std::memcpy(buf, s.data(), n);
        buf[n] = 0;
    }
    return int64_t(s.size() + 1);
}

int64_t vb_profile_processor_block(vb_model* m, int block, char* buf, size_t len) {
    std::string s;
    const int rc = guard([&] {
        need(m, "model");
        s = m->m->profile_block(block);
    });
    if (rc != VB_OK) return -rc;
    if (buf && len) {
        const size_t n = std::min(len - 1, s.size());
        std::memcpy(buf, s.data(), n);
        buf[n] = 0;
    }
    return int64_t(s.size() + 1);
}

int vb_build_csr(const int64_t* ei, int64_t E, const float* ea, int A, int64_t n_src, int64_t n_dst, int32_t* row_ptr,
                 int32_t* src, int32_t* edge_id, float* attr_csr) {
    return guard([&] {
        if (E < 0 || A < 1 || n_src < 0 || n_dst < 0) vb::fail(vb::kInvalidArgument, "bad graph sizes");
        need(row_ptr, "row_ptr");
        if (E > 0) need(ei, "edge_index"), need(ea, "edge_attr"), need(src, "src"), need(edge_id, "edge_id"),
            need(attr_csr, "attr_csr");
        vb::CsrGraph g = vb::build_csr_by_dst(ei, E, ea, A, n_src, n_dst);
        std::memcpy(row_ptr, g.row_ptr.data(), g.row_ptr.size() * sizeof(int32_t));
        if (E > 0) {
            std::memcpy(src, g.src.data(), g.src.size() * sizeof(int32_t));
            std::memcpy(edge_id, g.edge_id.data(), g.edge_id.size() * sizeof(int32_t));
            std::memcpy(attr_csr, g.attr.data(), g.attr.size() * sizeof(float));
        }
    });
}

int vb_pack_edges(const int32_t* src, const float* attr, int A, int64_t E, int round_fp16, void* out16) {
    return guard([&] {
        vb::CsrGraph g;
        g.n_edges = E;
        g.attr_dim = A;
        g.src.assign(src, src + E);
        g.attr.assign(attr, attr + E * A);
        auto p = vb::pack_edges(g, round_fp16 != 0);
        std::memcpy(out16, p.data(), p.size() * sizeof(vb::EdgeRec));
    });
}

int vb_rollout_update(float* window, int T, int64_t rows, int V_in, const float* y_own, const float* y_halo,
                      int64_t n_own, int V_out, const float* f, int F, const int8_t* kind, const int* src,
                      void* stream) {
    return guard([&] {
        need(window, "window"), need(kind, "kind"), need(src, "src");
        if (T < 1 || rows < 0 || V_in < 1 || V_out < 1 || F < 0 || n_own < 0 || n_own > rows)
            vb::fail(vb::kInvalidArgument, "rollout_update: bad sizes");
        vb::k::rollout_update(window, T, rows, V_in, y_own, y_halo, n_own, V_out, f, F, kind, src, S(stream));
    });
}

int vb_attention(int dtype, const int32_t* row_ptr, const void* edges, int64_t dst_lo, int64_t n_rows, const void* q,
                 int64_t ldq, const void* k, const void* v, int64_t ldkv, const void* xr, int64_t ldxr, void* out,
                 int64_t ldo, const float* w_e, int C, int heads, int head_dim, void* stream) {
    return guard([&] {
        auto run = [&](auto* tag) {
            using T = std::remove_pointer_t<decltype(tag)>;
            vb::k::AttnArgs<T> a;
            a.row_ptr = row_ptr, a.edges = static_cast<const vb::EdgeRec*>(edges), a.dst_lo = dst_lo;
            a.n_rows = n_rows, a.q = static_cast<const T*>(q), a.ldq = ldq, a.k = static_cast<const T*>(k);
            a.v = static_cast<const T*>(v), a.ldkv = ldkv, a.xr = static_cast<const T*>(xr), a.ldxr = ldxr;
            a.out = static_cast<T*>(out), a.ldo = ldo, a.w_e = w_e, a.C = C, a.heads = heads, a.head_dim = head_dim;
            vb::k::attention<T>(a, S(stream));
        };
        if (dtype == VB_PRECISION_FP32) run(static_cast<float*>(nullptr));
        else if (dtype == VB_PRECISION_FP16) run(static_cast<__half*>(nullptr));
        else vb::fail(vb::kInvalidArgument, "dtype");
    });
}

int vb_attention_rows(int dtype, const int32_t* row_ptr, const void* edges, const int32_t* rows, int64_t n_rows,
                      const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, const void* xr,
                      int64_t ldxr, void* out, int64_t ldo, const float* w_e, int C, int heads, int head_dim,
                      void* stream) {
    return guard([&] {
        need(row_ptr, "row_ptr"), need(rows, "rows"), need(w_e, "w_e");
        auto run = [&](auto* tag) {
            using T = std::remove_pointer_t<decltype(tag)>;
            vb::k::AttnArgs<T> a;
            a.row_ptr = row_ptr, a.edges = static_cast<const vb::EdgeRec*>(edges), a.dst_lo = 0, a.rows = rows;
            a.n_rows = n_rows, a.q = static_cast<const T*>(q), a.ldq = ldq, a.k = static_cast<const T*>(k);
            a.v = static_cast<const T*>(v), a.ldkv = ldkv, a.xr = static_cast<const T*>(xr), a.ldxr = ldxr;
            a.out = static_cast<T*>(out), a.ldo = ldo, a.w_e = w_e, a.C = C, a.heads = heads, a.head_dim = head_dim;
            vb::k::attention<T>(a, S(stream));
        };
        if (dtype == VB_PRECISION_FP32) run(static_cast<float*>(nullptr));
        else if (dtype == VB_PRECISION_FP16) run(static_cast<__half*>(nullptr));
        else vb::fail(vb::kInvalidArgument, "dtype");
    });
}

int vb_attention_split_noalloc(int dtype, const int32_t* row_ptr, const void* edges, int64_t dst_lo, int64_t n_rows,
                               const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, const void* xr,
                               int64_t ldxr, void* out, int64_t ldo, const float* w_e, int C, int heads, int head_dim,
                               int splits, void* stream) {
    return guard([&] {
        need(row_ptr, "row_ptr"), need(w_e, "w_e");
        auto run = [&](auto* tag) {
            using T = std::remove_pointer_t<decltype(tag)>;
            vb::k::AttnArgs<T> a;
            a.row_ptr = row_ptr, a.edges = static_cast<const vb::EdgeRec*>(edges), a.dst_lo = dst_lo;
            a.n_rows = n_rows, a.q = static_cast<const T*>(q), a.ldq = ldq, a.k = static_cast<const T*>(k);
            a.v = static_cast<const T*>(v), a.ldkv = ldkv, a.xr = static_cast<const T*>(xr), a.ldxr = ldxr;
            a.out = static_cast<T*>(out), a.ldo = ldo, a.w_e = w_e, a.C = C, a.heads = heads, a.head_dim = head_dim;
            vb::k::attention_split_noalloc<T>(a, splits, S(stream));
        };
        if (dtype == VB_PRECISION_FP32) run(static_cast<float*>(nullptr));
        else if (dtype == VB_PRECISION_FP16) run(static_cast<__half*>(nullptr));
        else vb::fail(vb::kInvalidArgument, "dtype");
    });
}

struct vb_tiles {
    vb::DeviceBuffer tiles, srcs, tedges, heavy, row_ptr, edges, blob;
    std::vector<int32_t> row0, row_end, heavy_rows;  // host copies: tile row ranges, heavy rows
    int kind = VB_TILES_SMEM;
    int64_t n_src = 0;
};

int vb_tiles_create(const int32_t* row_ptr, const int32_t* src, const float* attr, int A, int64_t n_src,
                    int64_t n_dst, int head_dim, vb_tiles** out) {
    return vb_tiles_create_kind(row_ptr, src, attr, A, n_src, n_dst, head_dim, VB_TILES_SMEM, out);
}

namespace {

vb::CsrGraph host_csr(const int32_t* row_ptr, const int32_t* src, const float* attr, int A, int64_t n_src,
                      int64_t n_dst) {
    vb::CsrGraph g;
    g.n_src = n_src, g.n_dst = n_dst, g.attr_dim = A;
    g.row_ptr.assign(row_ptr, row_ptr + n_dst + 1);
    g.n_edges = g.row_ptr.back();
    g.src.assign(src, src + g.n_edges);
    g.attr.assign(attr, attr + g.n_edges * A);
    return g;
}

// The tensor-core tiles' edges in the vb_tile_plan form {a0, a1, a2, slot (int bits)} in CSR order, decoded
// back from the tiles' record blocks (every masked fragment position of every chunk names its row and
// slot; the edge is the row's edge from that slot's source); a tiled edge no position names keeps
// NaN attributes and slot -1. Heavy rows: the packed record with their source. And each tile's
// {row0, nrows, src_off, nsrc}.
void tc_plan_export(const vb::CsrGraph& g, const vb::TcPlan& tp, int32_t* tiles4, float* edges) {
    if (tiles4)
        for (size_t i = 0; i < tp.tiles.size(); ++i)
            tiles4[4 * i] = tp.tiles[i].row0, tiles4[4 * i + 1] = tp.tiles[i].nrows,
                       tiles4[4 * i + 2] = tp.tiles[i].src_off, tiles4[4 * i + 3] = tp.tiles[i].nsrc;
    if (!edges) return;
    const auto packed = vb::pack_edges(g, true);
    std::memcpy(edges, packed.data(), packed.size() * sizeof(vb::EdgeRec));
    const int32_t none = -1;
    for (const vb::TcTile& t : tp.tiles)
        for (int64_t x = g.row_ptr[size_t(t.row0)]; x < g.row_ptr[size_t(t.row0 + t.nrows)]; ++x) {
            for (int k = 0; k < 3; ++k) edges[4 * x + k] = NAN;
            std::memcpy(edges + 4 * x + 3, &none, 4);
        }
    for (const vb::TcTile& t : tp.tiles) {
        const uint8_t* bl = tp.blob.data() + t.blob_off;
        for (int bk = 0; bk < (t.nrows + 15) / 16; ++bk) {
            const uint8_t* hd = bl + vb::kTcBlockOff + 32 * bk;
            for (int c = 0; c < hd[0]; ++c) {
                const int ci = hd[1] + c;
                const uint16_t* attr =
                    reinterpret_cast<const uint16_t*>(bl + t.attr_off + size_t(vb::kTcChunkAttr) * size_t(ci));
                for (int l = 0; l < 32; ++l)
                    for (int e = 0; e < 8; ++e) {
                        if (!((bl[vb::kTcMaskOff + 32 * ci + l] >> e) & 1)) continue;
                        const int row = 16 * bk + l / 4 + 8 * ((e >> 1) & 1);
                        const int32_t sl = 8 * hd[2 + 2 * c + (e >> 2)] + 2 * (l % 4) + (e & 1);
                        if (row >= t.nrows || sl >= t.nsrc) vb::fail(vb::kInternal, "tile plan: a masked position is outside its tile");
                        const int32_t source = tp.srcs[size_t(t.src_off + sl)];
                        int64_t x = g.row_ptr[size_t(t.row0 + row)];
                        while (x < g.row_ptr[size_t(t.row0 + row + 1)] && g.src[size_t(x)] != source) ++x;
                        if (x == g.row_ptr[size_t(t.row0 + row + 1)]) vb::fail(vb::kInternal, "tile plan: a masked position is not an edge");
                        for (int k = 0; k < 3; ++k)
                            edges[4 * x + k] = __half2float(__ushort_as_half(attr[24 * l + 2 * (3 * (e >> 1) + k) + (e & 1)]));
                        std::memcpy(edges + 4 * x + 3, &sl, 4);
                    }
            }
        }
    }
}

}  // namespace

int vb_tile_plan(const int32_t* row_ptr, const int32_t* src, const float* attr, int A, int64_t n_src, int64_t n_dst,
                 int kind, int64_t counts[3], int32_t* tiles4, int32_t* srcs, int32_t* heavy, float* edges) {
    return guard([&] {
        need(row_ptr, "row_ptr"), need(counts, "counts");
        if (kind != VB_TILES_SMEM && kind != VB_TILES_TC) vb::fail(vb::kInvalidArgument, "tiles kind");
        const vb::CsrGraph g = host_csr(row_ptr, src, attr, A, n_src, n_dst);
        if (kind == VB_TILES_TC) {
            const vb::TcPlan tp = vb::make_tc_tiles(g, vb::kTcAlignRows);
            counts[0] = int64_t(tp.tiles.size()), counts[1] = int64_t(tp.srcs.size());
            counts[2] = int64_t(tp.heavy.size());
            tc_plan_export(g, tp, tiles4, edges);
            if (srcs) std::copy(tp.srcs.begin(), tp.srcs.end(), srcs);
            if (heavy) std::copy(tp.heavy.begin(), tp.heavy.end(), heavy);
            return;
        }
        vb::TilePlan tp = vb::make_tiles(g, vb::k::tiled_max_src(), vb::k::tiled_max_rows(), vb::k::tiled_max_edges(),
                                         0, true);
        counts[0] = int64_t(tp.row0.size()), counts[1] = int64_t(tp.srcs.size()), counts[2] = int64_t(tp.heavy.size());
        if (tiles4)
            for (size_t i = 0; i < tp.row0.size(); ++i)
                tiles4[4 * i] = tp.row0[i], tiles4[4 * i + 1] = tp.nrows[i], tiles4[4 * i + 2] = tp.src0[i],
                           tiles4[4 * i + 3] = tp.nsrc[i];
        if (srcs) std::copy(tp.srcs.begin(), tp.srcs.end(), srcs);
        if (heavy) std::copy(tp.heavy.begin(), tp.heavy.end(), heavy);
        if (edges) std::memcpy(edges, tp.edges.data(), tp.edges.size() * sizeof(vb::EdgeRec));
    });
}

int vb_tiles_create_kind(const int32_t* row_ptr, const int32_t* src, const float* attr, int A, int64_t n_src,
                         int64_t n_dst, int head_dim, int kind, vb_tiles** out) {
    (void)head_dim;
    return guard([&] {
        need(row_ptr, "row_ptr"), need(out, "out");
        if (kind != VB_TILES_SMEM && kind != VB_TILES_TC) vb::fail(vb::kInvalidArgument, "tiles kind");
        const vb::CsrGraph g = host_csr(row_ptr, src, attr, A, n_src, n_dst);
        auto t = std::make_unique<vb_tiles>();
        t->kind = kind, t->n_src = n_src;
        auto up = [](vb::DeviceBuffer& b, const void* h, size_t n) {
            b.alloc(std::max<size_t>(n, 16));
            if (n) VB_CUDA(cudaMemcpy(b.get(), h, n, cudaMemcpyHostToDevice));
        };
        if (kind == VB_TILES_TC) {
            const vb::TcPlan tp = vb::make_tc_tiles(g, vb::kTcAlignRows);
            up(t->tiles, tp.tiles.data(), tp.tiles.size() * sizeof(vb::TcTile));
            up(t->srcs, tp.srcs.data(), tp.srcs.size() * 4);
            up(t->blob, tp.blob.data(), tp.blob.size());
            for (const vb::TcTile& x : tp.tiles) t->row0.push_back(x.row0), t->row_end.push_back(x.row0 + x.nrows);
            t->heavy_rows = tp.heavy;
        } else {
            vb::TilePlan tp = vb::make_tiles(g, vb::k::tiled_max_src(), vb::k::tiled_max_rows(),
                                             vb::k::tiled_max_edges(), 0, true);
            std::vector<int4> t4(tp.row0.size());
            for (size_t i = 0; i < t4.size(); ++i) t4[i] = make_int4(tp.row0[i], tp.nrows[i], tp.src0[i], tp.nsrc[i]);
            up(t->tiles, t4.data(), t4.size() * sizeof(int4));
            up(t->srcs, tp.srcs.data(), tp.srcs.size() * 4);
            up(t->tedges, tp.edges.data(), tp.edges.size() * sizeof(vb::EdgeRec));
            t->row0 = tp.row0;
            for (size_t i = 0; i < tp.row0.size(); ++i) t->row_end.push_back(tp.row0[i] + tp.nrows[i]);
            t->heavy_rows = tp.heavy;
        }
        up(t->heavy, t->heavy_rows.data(), t->heavy_rows.size() * 4);
        up(t->row_ptr, g.row_ptr.data(), g.row_ptr.size() * 4);
        auto packed = vb::pack_edges(g, true);
        up(t->edges, packed.data(), packed.size() * sizeof(vb::EdgeRec));
        *out = t.release();
    });
}

int vb_attention_tiled(vb_tiles* t, int64_t lo, int64_t n, const void* q, int64_t ldq, const void* k, const void* v,
                       int64_t ldkv, const void* xr, int64_t ldxr, void* out, int64_t ldo, const float* w_e, int C,
                       int heads, int head_dim, void* stream) {
    return guard([&] {
        need(t, "tiles"), need(q, "q"), need(k, "k"), need(v, "v"), need(xr, "xr"), need(out, "out"), need(w_e, "w_e");
        if (t->kind == VB_TILES_TC ? !vb::k::tc_attention_supported(C, heads, head_dim)
                                   : !vb::k::tiled_supported(C, head_dim))
            vb::fail(vb::kUnsupported, "tiled attention: unsupported layout");
        if (lo < 0 || n < 0 || lo + n > int64_t(t->row_ptr.bytes() / 4) - 1)
            vb::fail(vb::kInvalidArgument, "tiled attention: rows out of range");
        const auto t0 = std::lower_bound(t->row0.begin(), t->row0.end(), int32_t(lo));
        const auto t1 = std::lower_bound(t->row0.begin(), t->row0.end(), int32_t(lo + n));
        // the rows must not cut a tile: a tile writes all of its rows
        if (t1 > t0 && t->row_end[size_t(t1 - t->row0.begin()) - 1] > lo + n)
            vb::fail(vb::kInvalidArgument, "tiled attention: rows [dst_lo, dst_lo + n_rows) must end at a tile end");
        if (t0 != t->row0.end() && t0 != t->row0.begin() && t->row_end[size_t(t0 - t->row0.begin()) - 1] > lo)
            vb::fail(vb::kInvalidArgument, "tiled attention: dst_lo must start a tile");
        if (t->kind == VB_TILES_TC) {
            vb::k::TcArgs a;
            a.tiles = t->tiles.as<vb::TcTile>(), a.srcs = t->srcs.as<int32_t>(), a.blob = t->blob.as<uint8_t>();
            a.tile0 = int(t0 - t->row0.begin()), a.ntiles = int(t1 - t0), a.dst_lo = lo;
            a.q = static_cast<const __half*>(q), a.k = static_cast<const __half*>(k), a.v = static_cast<const __half*>(v);
            a.xr = static_cast<const __half*>(xr), a.out = static_cast<__half*>(out);
            a.ldq = ldq, a.ldkv = ldkv, a.ldxr = ldxr, a.ldo = ldo, a.n_q_rows = n;
            a.w_e = w_e, a.C = C, a.heads = heads, a.head_dim = head_dim;
            a.n_src = t->n_src;
            vb::k::attention_tc(a, S(stream));
        } else {
            vb::k::TileArgs a;
            a.tiles = t->tiles.as<int4>(), a.srcs = t->srcs.as<int32_t>(), a.edges = t->tedges.as<vb::EdgeRec>();
            a.row_ptr = t->row_ptr.as<int32_t>(), a.dst_lo = lo, a.tile0 = int(t0 - t->row0.begin());
            a.ntiles = int(t1 - t0);
            a.q = static_cast<const __half*>(q), a.k = static_cast<const __half*>(k), a.v = static_cast<const __half*>(v);
            a.xr = static_cast<const __half*>(xr), a.out = static_cast<__half*>(out);
            a.ldq = ldq, a.ldkv = ldkv, a.ldxr = ldxr, a.ldo = ldo, a.w_e = w_e, a.C = C, a.heads = heads;
            a.head_dim = head_dim;
            vb::k::attention_tiled(a, 1.4426950408889634f / std::sqrt(float(head_dim)), S(stream));
        }
        const auto h0 = std::lower_bound(t->heavy_rows.begin(), t->heavy_rows.end(), int32_t(lo));
        const auto h1 = std::lower_bound(t->heavy_rows.begin(), t->heavy_rows.end(), int32_t(lo + n));
        if (h1 > h0) {
            vb::k::AttnArgs<__half> g;
            g.row_ptr = t->row_ptr.as<int32_t>(), g.edges = t->edges.as<vb::EdgeRec>(), g.dst_lo = lo;
            g.rows = t->heavy.as<int32_t>() + (h0 - t->heavy_rows.begin()), g.n_rows = int64_t(h1 - h0);
            g.q = static_cast<const __half*>(q), g.ldq = ldq, g.k = static_cast<const __half*>(k);
            g.v = static_cast<const __half*>(v), g.ldkv = ldkv, g.xr = static_cast<const __half*>(xr), g.ldxr = ldxr;
            g.out = static_cast<__half*>(out), g.ldo = ldo, g.w_e = w_e, g.C = C, g.heads = heads, g.head_dim = head_dim;
            vb::k::attention<__half>(g, S(stream));
        }
    });
}

void vb_tiles_free(vb_tiles* t) { delete t; }

int vb_gemm(int dtype, int engine, const void* A, int64_t lda, const void* W, int64_t ldw, const void* bias, void* Y,
            int64_t ldy, const void* R, int64_t ldr, int64_t M, int64_t N, int64_t K, int epilogue, int gelu_tanh,
            void* stream) {
    return guard([&] {
        if (epilogue < 0 || epilogue > 2) vb::fail(vb::kInvalidArgument, "epilogue");
        auto fill = [&](auto& a, auto* tag) {
            using T = std::remove_pointer_t<decltype(tag)>;
            a.A = static_cast<const T*>(A), a.lda = lda, a.W = static_cast<const T*>(W), a.ldw = ldw;
            a.bias = static_cast<const T*>(bias), a.C = static_cast<T*>(Y), a.ldc = ldy;
            a.R = static_cast<const T*>(R), a.ldr = ldr, a.M = M, a.N = N, a.K = K, a.epi = epilogue;
            a.gelu_tanh = gelu_tanh != 0;
        };
        if (dtype == VB_PRECISION_FP32) {
            if (engine == 2) vb::fail(vb::kUnsupported, "tensor-core gemm takes fp16 only");
            vb::k::GemmArgs<float> a;
            fill(a, static_cast<float*>(nullptr));
            vb::k::gemm_simt<float>(a, S(stream));
        } else if (dtype == VB_PRECISION_FP16) {
            vb::k::GemmArgs<__half> a;
            fill(a, static_cast<__half*>(nullptr));
            if (engine != 1 && vb::tc::supported(a)) vb::tc::gemm(a, S(stream));
            else if (engine == 2) vb::fail(vb::kUnsupported, "operands not aligned for the tensor-core gemm");
            else vb::k::gemm_simt<__half>(a, S(stream));
        } else {
            vb::fail(vb::kInvalidArgument, "dtype");
        }
    });
}

int vb_ln_segment_width(int64_t N) { return vb::tc::stats_segw(N); }

int vb_gemm_ln(const void* A, int64_t lda, const void* W, int64_t ldw, const void* bias, void* Y, int64_t ldy,
               const void* R, int64_t ldr, int64_t M, int64_t N, int64_t K, int epilogue, int gelu_tanh, float* st_out,
               const float* st_in, const float* colsum, int nseg_in, int segw_in, float eps, void* stream) {
    return guard([&] {
        if (epilogue < 0 || epilogue > 2) vb::fail(vb::kInvalidArgument, "epilogue");
        vb::k::GemmArgs<__half> a;
        a.A = static_cast<const __half*>(A), a.lda = lda, a.W = static_cast<const __half*>(W), a.ldw = ldw;
        a.bias = static_cast<const __half*>(bias), a.C = static_cast<__half*>(Y), a.ldc = ldy;
        a.R = static_cast<const __half*>(R), a.ldr = ldr, a.M = M, a.N = N, a.K = K, a.epi = epilogue;
        a.gelu_tanh = gelu_tanh != 0;
        a.st_out = reinterpret_cast<float2*>(st_out), a.st_in = reinterpret_cast<const float2*>(st_in);
        a.colsum = colsum, a.nseg_in = nseg_in, a.segw_in = segw_in, a.eps = eps;
        if (!vb::tc::supported(a)) vb::fail(vb::kUnsupported, "gemm_ln: operands or LayerNorm arguments not supported");
        vb::tc::gemm(a, S(stream));
    });
}

int vb_fold_layernorm(void* W, int64_t ldw, int64_t N, int K, const float* g, const float* be, void* bias,
                      float* colsum, void* stream) {
    return guard([&] {
        if (!W || !g || !bias || !colsum || K < 1 || ldw < K) vb::fail(vb::kInvalidArgument, "fold_layernorm");
        vb::k::fold_layernorm(static_cast<__half*>(W), ldw, N, K, g, be, static_cast<__half*>(bias), colsum, S(stream));
    });
}

int vb_row_seg_stats(const void* x, int64_t ldx, int64_t rows, int C, int segw, float* st, void* stream) {
    return guard([&] {
        vb::k::row_seg_stats(static_cast<const __half*>(x), ldx, rows, C, segw, reinterpret_cast<float2*>(st), S(stream));
    });
}

int vb_layernorm(int dtype, const void* x, int64_t ldx, const float* w, const float* b, void* y, int64_t ldy,
                 int64_t rows, int C, float eps, void* stream) {
    return guard([&] {
        if (dtype == VB_PRECISION_FP32)
            vb::k::layernorm<float>(static_cast<const float*>(x), ldx, w, b, static_cast<float*>(y), ldy, rows, C, eps,
                                    S(stream));
        else if (dtype == VB_PRECISION_FP16)
            vb::k::layernorm<__half>(static_cast<const __half*>(x), ldx, w, b, static_cast<__half*>(y), ldy, rows, C,
                                     eps, S(stream));
        else vb::fail(vb::kInvalidArgument, "dtype");
    });
}

int vb_add_layernorm(int dtype, const void* a, const void* r, void* out1, const float* w, const float* b, void* ln,
                     int64_t ld, int64_t rows, int C, float eps, void* stream) {
    return guard([&] {
        if (dtype == VB_PRECISION_FP32)
            vb::k::add_layernorm<float>(static_cast<const float*>(a), static_cast<const float*>(r),
                                        static_cast<float*>(out1), w, b, static_cast<float*>(ln), ld, rows, C, eps,
                                        S(stream));
        else if (dtype == VB_PRECISION_FP16)
            vb::k::add_layernorm<__half>(static_cast<const __half*>(a), static_cast<const __half*>(r),
                                         static_cast<__half*>(out1), w, b, static_cast<__half*>(ln), ld, rows, C, eps,
                                         S(stream));
        else vb::fail(vb::kInvalidArgument, "dtype");
    });
}

}  // extern "C"
