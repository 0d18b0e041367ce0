// Engine<T>: loading, buffers and the GraphTransformer forward pass on one B200.
//
// The op sequence is the reference's (CPU oracle backend_cpu.cpp:297-537; CUDA engine
// backend_cuda.cu:523-667), restructured for this GPU:
//   * residual adds and GELU are fused into the epilogue of the GEMM that produces them
//     (proj + residual, mlp1 + GELU, mlp2 + residual), keeping the autocast roundings
//     T(T(acc + b) + r) and T(gelu(T(acc + b)));
//   * q|k|v|self (processor), q|self and k|v (mappers) are one stacked GEMM each;
//   * the edge projection is folded into the attention kernel (no [E, C] tensor);
//   * with 180 GB of HBM the decoder normally runs all data rows as one chunk.
#include <cuda_fp16.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "comm.h"
#include "common.h"
#include "config.h"
#include "engine.h"
#include "gemm_tc.cuh"
#include "graph.h"
#include "kernels.cuh"
#include "params.h"
#include "safetensors.h"
#include "shard.h"

namespace vb {

namespace {

int64_t env_int(const char* name, int64_t dflt) {
    const char* v = std::getenv(name);
    return v && *v ? std::atoll(v) : dflt;
}

// Which graphs run the shared-memory-staged tiled attention (fp16): VB_ATT_TILED = "1" / "all" (every
// graph), "0" / "none", or a comma-separated list of graph names (enc, proc, dec); unset: `dflt`.
// measured on C1 (B200): tiled 5.2 ms vs gather 12.4 ms on the decoder (3 edges per row, heavily
// shared sources), equal on the processor, gather ahead on the encoder (35 edges per row)
constexpr const char* kTiledDefault = "dec";
// Which graphs run the tile-sparse tensor-core attention (fp16, head_dim 64; attention_tc.cu): VB_ATT_TC,
// the same forms; it takes precedence over VB_ATT_TILED. Default: the processor graph, where it measured
// 1.25 ms per C2 block against 1.57 ms for the gather kernel (1.66 against 2.16 ms per block inside the
// C1 step, 167.9 against 173.8 ms per step). A graph whose tiles would not restart on the 64-row grid
// of a decoder chunk keeps its other kernel.
constexpr const char* kTcDefault = "proc";
bool graph_listed(const char* env, const std::string& graph, const char* dflt) {
    const char* v = std::getenv(env);
    const std::string s = v && *v ? v : dflt;
    if (s == "1" || s == "all") return true;
    if (s == "0" || s == "none") return false;
    size_t b = 0;
    while (b <= s.size()) {
        size_t e = s.find(',', b);
        if (e == std::string::npos) e = s.size();
        if (s.compare(b, e - b, graph) == 0) return true;
        b = e + 1;
    }
    return false;
}
bool tiled_for(const std::string& graph, const char* dflt) { return graph_listed("VB_ATT_TILED", graph, dflt); }
bool tc_for(const std::string& graph) { return graph_listed("VB_ATT_TC", graph, kTcDefault); }
// Which graphs' gather launches visit destinations in source order (VB_ATT_ORDER, same forms).
constexpr const char* kOrderDefault = "enc";

// Load-stage timer: VB_LOAD_TIMING=1 prints the seconds of each stage of a model load to stderr.
struct LoadTimer {
    bool on = env_int("VB_LOAD_TIMING", 0) != 0;
    std::chrono::steady_clock::time_point t = std::chrono::steady_clock::now();
    void mark(const char* stage) {
        if (!on) return;
        const auto now = std::chrono::steady_clock::now();
        std::fprintf(stderr, "varda_b200 load: %-28s %.3f s\n", stage, std::chrono::duration<double>(now - t).count());
        t = now;
    }
};

struct GraphDev {
    std::string name;
    DeviceBuffer row_ptr, edges;
    int64_t n_src = 0, n_dst = 0, n_edges = 0;
    int max_degree = 0;
    const int32_t* rp() const { return row_ptr.as<int32_t>(); }
    const EdgeRec* ed() const { return edges.as<EdgeRec>(); }
    // destination tiles of the shared-memory-staged attention (fp16), or of the tensor-core attention
    // (tc: TcTile descriptors in `tiles`, record blocks in `tblob`), and the heavy rows
    bool tiled = false, tc = false;
    DeviceBuffer tiles, srcs, tedges, heavy, tblob;
    std::vector<int32_t> tile_row0, heavy_rows;  // host copies, to pick a chunk's tiles
    // wide rows (more than kWideDeg edges, VB_ATT_WIDE_DEG; 0 disables) cut into parts of kPartEdges
    // edges (VB_ATT_PART_EDGES), run by the split kernels over a scratch of one partial record per
    // part, so one row's edges no longer run serially on one warp; the other rows go to the gather
    // kernel. A guard for extreme degrees: on the C1 encoder (rows of up to 1,456 edges) splitting at
    // 128 measured 9.6 ms against 5.3 ms for the gather kernel alone, whose per-edge rate dominates.
    bool wide = false;
    DeviceBuffer light, wide_dev, part0_dev, parts, scratch;
    // destination visiting order for a whole-graph gather launch (VB_ATT_ORDER; empty: index order):
    // rows sorted by their smallest source, so rows that gather the same sources run close together
    DeviceBuffer order;
    std::vector<int32_t> light_rows, wide_rows, part0;  // host copies (sorted rows; part prefix)
};
constexpr int kWideDeg = 2048, kPartEdges = 64;

}  // namespace

template <class T>
class Engine final : public Model {
public:
    Engine(const std::string& path, const Options& o);
    ~Engine() override;

    void predict_step(const float* x, float* y, HookFn hook, void* user) override;
    // device tensors hold this rank's rows: x/xn (T_in, Gx, V_in) = own data rows then the encoder's
    // halo rows; yn/y (T_out, Gl, V_out) = own data rows (all rows on one GPU)
    int64_t input_numel() const override { return int64_t(T_in_) * Gx_ * V_in_; }
    int64_t output_numel() const override { return int64_t(T_out_) * Gl_ * V_out_; }
    void normalise(const float* x, float* xn, cudaStream_t s) override {
        k::normalise(x, mul_in_.as<float>(), add_in_.as<float>(), xn, input_numel(), V_in_, s);
    }
    void forward_normalised(const float* xn, float* yn, cudaStream_t s) override { forward(xn, yn, s, nullptr); }
    void denormalise(const float* yn, float* y, cudaStream_t s) override {
        k::denormalise(yn, add_out_.as<float>(), mul_out_.as<float>(), y, output_numel(), V_out_, s);
    }
    // sharded: x's encoder-halo rows are filled from their owners first (the caller fills own rows)
    void predict_step_device(const float* x, float* y, cudaStream_t s) override {
        exchange_input(const_cast<float*>(x), s);
        normalise(x, xn_, s);
        forward(xn_, yn_, s, nullptr);
        denormalise(yn_, y, s);
    }
    void prepare() override;
    void use_high_priority_stream() override;
    float* device_input() override { return x_dev_; }
    const float* device_output() const override { return y_dev_; }
    cudaStream_t stream() const override { return stream_; }
    void enqueue_predict() override;
    int device() const override { return dev_; }
    size_t weight_bytes() const override { return weight_bytes_; }
    size_t activation_bytes() const override { return act_bytes_; }
    int64_t decoder_chunk_rows() const override { return dec_rows_; }
    void sizes(int64_t o[8]) const override {
        o[0] = T_in_, o[1] = G_, o[2] = V_in_, o[3] = T_out_, o[4] = V_out_, o[5] = H_, o[6] = C_, o[7] = n_proc_;
    }
    void data_range(int64_t* lo, int64_t* hi) const override { *lo = plan_.g_lo, *hi = plan_.g_hi; }
    void hidden_range(int64_t* lo, int64_t* hi) const override { *lo = plan_.h_lo, *hi = plan_.h_hi; }
    void processor_block(int block, const float* z_in, float* z_out, int repeats, float* device_ms) override;
    std::string profile_forward() override;
    std::string profile_block(int block) override;
    template <class F> std::string profiled(F body);
    void rollout(const float* x0, int n_steps, const float* forcings, float* y, bool constants_oldest, StepFn cb,
                 void* user, float* step_ms) override;

private:
    struct HookSink;
    // ---- profiling (eager runs only): an event pair around every launch
    struct ProfRec {
        std::string name;
        cudaEvent_t a, b;
        double flop, bytes;
    };
    std::vector<ProfRec>* prof_ = nullptr;
    struct Span {
        Engine* e;
        cudaStream_t s;
        Span(Engine* en, cudaStream_t st, std::string name, double flop, double bytes) : e(en), s(st) {
            if (!e->prof_) return;
            ProfRec r{std::move(name), nullptr, nullptr, flop, bytes};
            VB_CUDA(cudaEventCreate(&r.a));
            VB_CUDA(cudaEventCreate(&r.b));
            VB_CUDA(cudaEventRecord(r.a, s));
            e->prof_->push_back(r);
        }
        ~Span() {
            if (e->prof_) cudaEventRecord(e->prof_->back().b, s);
        }
    };
    void ln(const T* x, const Affine& n, T* y, int64_t rows, cudaStream_t s) {
        Span sp(this, s, "layernorm", 0, double(rows) * C_ * 2 * sizeof(T));
        k::layernorm<T>(x, C_, n.g(), n.b(), y, C_, rows, C_, eps_, s);
    }
    CsrGraph read_graph(SafeTensorsFile& f, const std::string& g, int64_t n_src, int64_t n_dst);
    GraphDev upload_graph(const CsrGraph& csr, const std::string& name, int64_t chunk_rows);
    DeviceBuffer upload(const void* h, size_t bytes);
    T* act(size_t elems);
    float* actf(size_t elems);

    // st_out: write the output rows' LayerNorm segment records there; st_in: L has a LayerNorm folded in
    // and x's rows have their records there (both only with fold_)
    void linear(const Dense<T>& L, const T* x, int64_t ldx, T* y, int64_t ldy, int64_t M, cudaStream_t s,
                int epi = k::kEpiBias, const T* R = nullptr, int64_t ldr = 0, float2* st_out = nullptr,
                const float2* st_in = nullptr);
    // y = L(LN(x)) for x [M, C]: when L has the LN folded in, L on x and x's records st; else the LN
    // kernel into xh (which may be x), then L
    void ln_linear(const Affine& n, const Dense<T>& L, const T* x, const float2* st, T* xh, T* y, int64_t ldy,
                   int64_t M, cudaStream_t s, int epi = k::kEpiBias) {
        if (L.cs()) return linear(L, x, C_, y, ldy, M, s, epi, nullptr, 0, nullptr, st);
        ln(x, n, xh, M, s);
        linear(L, xh, C_, y, ldy, M, s, epi);
    }
    // the records of rows [0, rows) of x when no GEMM epilogue wrote them
    void row_stats(const T* x, int64_t rows, float2* st, cudaStream_t s);
    void attention(const GraphDev& g, const AttnLayer<T>& b, int64_t lo, int64_t n, const T* q, int64_t ldq, const T* kk,
                   const T* v, int64_t ldkv, const T* xr, int64_t ldxr, T* out, cudaStream_t s);
    void forward(const float* xn, float* yn, cudaStream_t s, HookSink* hk);
    // pieces of forward(), in its order; the pipelined host path runs them around chunked copies
    void enc_source(const float* xn, int64_t slot_rows, int64_t r0, int64_t n, cudaStream_t s, HookSink* hk);
    void enc_dest_pre(cudaStream_t s, HookSink* hk);
    bool middle(cudaStream_t s, HookSink* hk);
    void proc_block(int i, const T* z_in, T* z_out, bool overlap, cudaStream_t s);
    // processor_block(): fp32 [H, C] host-copy staging and the events around its runs
    DeviceBuffer blk_stage_;
    cudaEvent_t blk_ev_[2] = {nullptr, nullptr};
    void dec_chunk(int64_t lo, int64_t n, cudaStream_t s, HookSink* hk, bool& halo_pending, float* h_emb, float* h_bo);
    void output_rows(const float* xn, float* yn, int64_t lo, int64_t n, cudaStream_t s, float* pre_bound);
    cudaGraphExec_t capture(const std::function<void(cudaStream_t)>& body, cudaStream_t s);
    bool capture_graph(cudaStream_t s);
    void upload_input(const float* x, cudaStream_t s);

    Config cfg_;
    Options opts_;
    int dev_ = 0;
    cudaStream_t stream_ = nullptr;
    bool use_tc_ = false;
    // LayerNorm folded into the Linear after it (fp16 tensor-core path): an LN's statistics are segment
    // records of its input rows, written by the epilogue of the GEMM that produced them (or by
    // row_stats), and the Linear's weights carry the LN's affine parameters. VB_LN_FOLD: 1 (default) the
    // LNs before the bias-epilogue Linears (ln_src, ln_dst, out_norm); 2 also ln_mlp, whose GELU GEMM's
    // epilogue bounds it already (its fold measured slower than the LN kernel it removes); 0 none.
    // stA_: the records of a block's input (and of the decoder's emb_dst and block output), stB_: of its
    // out1 (fold_mlp_); nseg_ records of segw_ columns per row.
    bool fold_ = false, fold_mlp_ = false;
    float2 *stA_ = nullptr, *stB_ = nullptr;
    int nseg_ = 0, segw_ = 0;
    // the dynamic tile order's counters of this model's GEMMs and tensor-core attention launches (all on
    // its stream, one at a time): words 0-1 and 2-3 of gemm_sched_
    DeviceBuffer gemm_sched_;
    unsigned* sched_ = nullptr;
    unsigned* att_sched_ = nullptr;
    int C_ = 0, heads_ = 0, hd_ = 0, mlp_ = 0, n_proc_ = 0, T_in_ = 0, T_out_ = 0, V_in_ = 0, V_out_ = 0, V_dec_ = 0;
    int A_node_ = 0, F_ = 0;
    int64_t ldF_ = 0, ldA_ = 0, ldVo_ = 0;
    int64_t G_ = 0, H_ = 0;
    float eps_ = 0;
    bool gelu_tanh_ = false;

    Dense<T> enc_emb_src_, enc_emb_dst_, dec_emb_dst_, dec_out_proj_;
    Affine dec_out_norm_;
    AttnLayer<T> enc_, dec_;
    std::vector<AttnLayer<T>> proc_;
    GraphDev g_enc_, g_proc_, g_dec_;
    DeviceBuffer mul_in_, add_in_, mul_out_, add_out_, res_src_, bounds_, bidx_;
    int n_bounds_ = 0;
    DeviceBuffer d_attr_, h_attr_;
    std::vector<float> h_attr_host_;
    size_t weight_bytes_ = 0;

    std::vector<DeviceBuffer> acts_;
    size_t act_bytes_ = 0;
    float *x_dev_ = nullptr, *xn_ = nullptr, *yn_ = nullptr, *y_dev_ = nullptr;
    T *x_data_ = nullptr, *region_ = nullptr, *dec_out_ = nullptr;
    T *z_enc_ = nullptr, *zA_ = nullptr, *zB_ = nullptr, *xh_ = nullptr, *qkvs_ = nullptr, *sbuf_ = nullptr;
    T *out1_ = nullptr, *hbuf_ = nullptr;
    int64_t dec_rows_ = 0;

    DeviceBuffer hook_stage_, hook_xsrc_, hook_prebound_;
    bool ran_eager_ = false, graph_failed_ = false;
    cudaGraphExec_t graph_exec_ = nullptr;

    // ---- destination partition (world == 1: the identity, no halos)
    ShardPlan plan_;
    int64_t Hl_ = 0, Gl_ = 0, Gx_ = 0, n_eh_ = 0, n_ph_ = 0, n_dh_ = 0;
    int64_t El_ = 0;  // the encoder's destination rows (= Hl_ unless the encoder is split on its own)
    std::unique_ptr<Comm> comm_;
    // encoder split: the encoder's output rows [e_lo, e_hi) go to their processor owners (one
    // contiguous row range per peer each way, in elements of C; own rows by a device copy)
    struct EncMove {
        bool on = false;
        std::vector<int64_t> send_off, send_cnt, recv_off, recv_cnt;
        int64_t self_src = 0, self_dst = 0, self_rows = 0;
    } emove_;
    void enc_redistribute(const T* src, T* dst, cudaStream_t s);
    struct Xchg {  // one halo exchange: pack own K|V rows per peer, send/recv, (unpack)
        DeviceBuffer send_idx;  // local ids of the rows sent, grouped by peer
        std::vector<int64_t> send_off, send_cnt, recv_off, recv_cnt;  // in elements
        int64_t n_send = 0, n_recv = 0;                                // in rows
    };
    Xchg xp_, xd_;
    // overlap (sharded, graph / eager runs without profiling): the processor's K|V halo exchange runs
    // on cs_ while the attention of the interior rows (no remote source) runs; the boundary rows follow
    cudaStream_t cs_ = nullptr;
    cudaEvent_t ev_kv_ = nullptr, ev_halo_ = nullptr;
    // pipelined host I/O (one GPU, no hook): the host -> device copy of x in row chunks on cio_ while the
    // encoder's source side runs on the chunks already there, and the decoder in row chunks whose
    // outputs go back on cio_ while the next chunk runs; each compute piece is a CUDA graph
    struct IoSeg {  // one piece of the pipelined step: a graph of `body`, or `body` run eagerly
        std::function<void(cudaStream_t)> body;
        cudaGraphExec_t graph = nullptr;
    };
    struct IoPipe {
        bool on = false, ready = false;
        int64_t in_rows = 0, dec_rows = 0;  // input chunk rows; decoder chunk rows (never straddle a tile)
        cudaStream_t cio = nullptr;
        cudaEvent_t start = nullptr;
        std::vector<cudaEvent_t> in_done, out_done;
        IoSeg pre, halo, mid;
        std::vector<IoSeg> src, dec;
    } io_;
    void io_run(IoSeg& g, cudaStream_t s) {
        if (g.graph) VB_CUDA(cudaGraphLaunch(g.graph, s));
        else if (g.body) g.body(s);
    }
    void io_setup();
    void io_release();
    void predict_pipelined(const float* x, float* y);
    DeviceBuffer proc_inner_, proc_outer_;
    int64_t n_inner_ = 0, n_outer_ = 0;
    // the same split for the tensor-core processor attention: its tiles reordered, those with no remote
    // source first (n_tc_inner_ of them); its heavy rows by the row split
    DeviceBuffer proc_tc_tiles_, proc_heavy_inner_, proc_heavy_outer_;
    int n_tc_inner_ = 0, n_tc_tiles_ = 0;
    int64_t n_heavy_inner_ = 0, n_heavy_outer_ = 0;
    void proc_attention_part(const AttnLayer<T>& b, bool boundary, cudaStream_t s);
    void attention_rows(const GraphDev& g, const AttnLayer<T>& b, const DeviceBuffer& rows, int64_t n, const T* q,
                        int64_t ldq, const T* kk, const T* v, int64_t ldkv, const T* xr, int64_t ldxr, T* out,
                        cudaStream_t s);
    T *xsend_ = nullptr, *xrecv_ = nullptr;
    // the encoder's halo input rows (all T_in slots) from their owners, at the start of every forward
    Xchg xx_;
    float *xx_send_ = nullptr, *xx_recv_ = nullptr;
    void exchange_input(float* x, cudaStream_t s);
    // send lists in local row ids (global id - lo); offsets and counts in elements of `row` per row
    void setup_exchange(Xchg& x, const HaloPlan& h, int64_t lo, int64_t row);

    // ---- rollout (set up by the first rollout call)
    struct Roll {
        bool ready = false;
        int F = 0;
        int oldest = -1;                     // constant source the kind array was built for
        std::vector<int8_t> kind;            // [V_in] 0 kept, 1 prognostic, 2 forcing (3: kept from the oldest slot)
        DeviceBuffer d_kind, d_src, f[2], y[2];
        float *hy[2] = {nullptr, nullptr}, *hf[2] = {nullptr, nullptr};
        cudaStream_t d2h = nullptr, h2d = nullptr;
        cudaEvent_t up[2] = {nullptr, nullptr}, down[2] = {nullptr, nullptr};
        std::vector<cudaEvent_t> beg, end;
        cudaGraphExec_t graph[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};  // [parity][with update]
        bool graph_failed = false;
    } ro_;
    void rollout_setup();
    void rollout_body(int p, bool update, cudaStream_t s);
    void rollout_release();
    void exchange(Xchg& x, const T* src, int64_t lds, T* dst, int64_t ldd, bool direct, cudaStream_t s);
};

// ====================================================================== hook

// Delivers activations to the caller's hook (eager runs only) as host fp32, contiguous. A device
// tensor [rows, cols] (row stride ld, element type U) is converted to fp32 on the device into a staging
// buffer in slabs of whole rows, alternating between the buffer's two halves, each slab copied to the
// host behind its conversion on the same stream; one synchronisation at the end.
template <class T>
struct Engine<T>::HookSink {
    Engine& e;
    HookFn fn;
    void* user;
    cudaStream_t s;
    static constexpr int64_t kStageFloats = int64_t(1) << 24;

    void emit_host(const std::string& key, const float* host, std::vector<int64_t> shape) {
        fn(key.c_str(), host, shape.data(), int(shape.size()), user);
    }
    // rows [0, rows) of the device tensor into dst rows [row0, row0 + rows)
    template <class U> void to_host(const U* d, int64_t ld, int64_t rows, int64_t cols, float* dst, int64_t row0 = 0) {
        if (!e.hook_stage_.get()) e.hook_stage_.alloc(size_t(kStageFloats) * sizeof(float));
        const int64_t slab = std::max<int64_t>(1, kStageFloats / 2 / std::max<int64_t>(cols, 1));
        for (int64_t r = 0, i = 0; r < rows; r += slab, ++i) {
            const int64_t n = std::min(slab, rows - r);
            float* half = e.hook_stage_.as<float>() + (i & 1) * (kStageFloats / 2);
            k::convert_2d<U, float>(d + r * ld, ld, half, cols, n, cols, s);
            VB_CUDA(cudaMemcpyAsync(dst + (row0 + r) * cols, half, size_t(n * cols) * sizeof(float),
                                    cudaMemcpyDeviceToHost, s));
        }
        VB_CUDA(cudaStreamSynchronize(s));
    }
    template <class U> void emit(const std::string& key, const U* d, int64_t ld, int64_t rows, int64_t cols,
                                 std::vector<int64_t> shape) {
        std::vector<float> host(size_t(rows * cols));
        to_host(d, ld, rows, cols, host.data());
        emit_host(key, host.data(), std::move(shape));
    }
};

// ====================================================================== loading

template <class T>
DeviceBuffer Engine<T>::upload(const void* h, size_t bytes) {
    DeviceBuffer b(bytes);
    // an empty host vector (null data) still gets a zeroed placeholder allocation
    if (bytes && h) VB_CUDA(cudaMemcpy(b.get(), h, bytes, cudaMemcpyHostToDevice));
    else if (bytes) VB_CUDA(cudaMemset(b.get(), 0, bytes));
    weight_bytes_ += bytes;
    return b;
}

template <class T>
CsrGraph Engine<T>::read_graph(SafeTensorsFile& f, const std::string& g, int64_t n_src, int64_t n_dst) {
    const TensorView& ei = f.take("graph." + g + ".edge_index");
    const TensorView& ea = f.take("graph." + g + ".edge_attr");
    if (ea.shape.size() != 2 || ea.shape[1] != cfg_.edge_attr_dim)
        fail(kFormat, ea.name + ": expected [E, " + std::to_string(cfg_.edge_attr_dim) + "], got " + ea.shape_str());
    return build_csr_by_dst(ei, ea, n_src, n_dst);
}

template <class T>
GraphDev Engine<T>::upload_graph(const CsrGraph& csr, const std::string& name, int64_t chunk_rows) {
    std::vector<EdgeRec> packed = pack_edges(csr, !std::is_same<T, float>::value);
    GraphDev d;
    d.name = name;
    const bool half = std::is_same<T, __half>::value;
    // the tensor-core tiles restart every kTcAlignRows rows; a chunked graph needs chunks on that grid
    const bool tc = half && k::tc_attention_supported(C_, heads_, hd_) && tc_for(name) &&
                    (chunk_rows <= 0 || chunk_rows % kTcAlignRows == 0);
    if (tc) {
        const TcPlan tp = make_tc_tiles(csr, kTcAlignRows);
        d.tiled = true, d.tc = true;
        d.tiles = upload(tp.tiles.data(), std::max<size_t>(1, tp.tiles.size()) * sizeof(TcTile));
        d.srcs = upload(tp.srcs.data(), std::max<size_t>(1, tp.srcs.size()) * sizeof(int32_t));
        d.tblob = upload(tp.blob.data(), std::max<size_t>(16, tp.blob.size()));
        d.heavy = upload(tp.heavy.data(), std::max<size_t>(1, tp.heavy.size()) * sizeof(int32_t));
        for (const TcTile& t : tp.tiles) d.tile_row0.push_back(t.row0);
        d.heavy_rows = tp.heavy;
    } else if (half && k::tiled_supported(C_, hd_) && tiled_for(name, kTiledDefault)) {
        TilePlan tp = make_tiles(csr, k::tiled_max_src(), k::tiled_max_rows(), k::tiled_max_edges(), chunk_rows, true);
        std::vector<int4> t4(tp.row0.size());
        for (size_t i = 0; i < t4.size(); ++i) t4[i] = make_int4(tp.row0[i], tp.nrows[i], tp.src0[i], tp.nsrc[i]);
        d.tiled = true;
        d.tiles = upload(t4.data(), std::max<size_t>(1, t4.size()) * sizeof(int4));
        d.srcs = upload(tp.srcs.data(), std::max<size_t>(1, tp.srcs.size()) * sizeof(int32_t));
        d.tedges = upload(tp.edges.data(), std::max<size_t>(1, tp.edges.size()) * sizeof(EdgeRec));
        d.heavy = upload(tp.heavy.data(), std::max<size_t>(1, tp.heavy.size()) * sizeof(int32_t));
        d.tile_row0 = tp.row0;
        d.heavy_rows = tp.heavy;
    }
    const int64_t wide_deg = env_int("VB_ATT_WIDE_DEG", kWideDeg), part_edges = env_int("VB_ATT_PART_EDGES", kPartEdges);
    if (!d.tiled && wide_deg > 0 && part_edges > 0 && csr.max_degree() > wide_deg) {
        std::vector<int4> pt;
        for (int64_t r = 0; r < csr.n_dst; ++r) {
            const int32_t b = csr.row_ptr[size_t(r)], e = csr.row_ptr[size_t(r + 1)];
            if (e - b <= wide_deg) {
                d.light_rows.push_back(int32_t(r));
                continue;
            }
            d.wide_rows.push_back(int32_t(r));
            d.part0.push_back(int32_t(pt.size()));
            for (int32_t x = b; x < e; x += int32_t(part_edges))
                pt.push_back(make_int4(int32_t(r), x, std::min(e, x + int32_t(part_edges)), 0));
        }
        d.part0.push_back(int32_t(pt.size()));
        d.wide = true;
        d.light = upload(d.light_rows.data(), std::max<size_t>(1, d.light_rows.size()) * sizeof(int32_t));
        d.wide_dev = upload(d.wide_rows.data(), d.wide_rows.size() * sizeof(int32_t));
        d.part0_dev = upload(d.part0.data(), d.part0.size() * sizeof(int32_t));
        d.parts = upload(pt.data(), pt.size() * sizeof(int4));
        d.scratch.alloc(pt.size() * size_t(k::attention_parts_record(C_, heads_)) * sizeof(float));
        act_bytes_ += d.scratch.bytes();
    }
    if (!d.tiled && !d.wide && graph_listed("VB_ATT_ORDER", name, kOrderDefault) && csr.n_dst > 0) {
        std::vector<int64_t> key(size_t(csr.n_dst));
        for (int64_t r = 0; r < csr.n_dst; ++r) {
            int64_t k = csr.n_src + r;  // rows without edges go last
            for (int32_t e = csr.row_ptr[size_t(r)]; e < csr.row_ptr[size_t(r + 1)]; ++e) k = std::min<int64_t>(k, csr.src[size_t(e)]);
            key[size_t(r)] = k;
        }
        std::vector<int32_t> ord(size_t(csr.n_dst));
        for (int64_t r = 0; r < csr.n_dst; ++r) ord[size_t(r)] = int32_t(r);
        std::stable_sort(ord.begin(), ord.end(), [&](int32_t a, int32_t b) { return key[size_t(a)] < key[size_t(b)]; });
        d.order = upload(ord.data(), ord.size() * sizeof(int32_t));
    }
    d.row_ptr = upload(csr.row_ptr.data(), csr.row_ptr.size() * sizeof(int32_t));
    d.edges = upload(packed.data(), std::max<size_t>(1, packed.size()) * sizeof(EdgeRec));
    d.n_src = csr.n_src;
    d.n_dst = csr.n_dst;
    d.n_edges = csr.n_edges;
    d.max_degree = csr.max_degree();
    return d;
}

template <class T>
void Engine<T>::setup_exchange(Xchg& x, const HaloPlan& h, int64_t lo, int64_t row) {
    const int W = plan_.world;
    x.send_off.assign(size_t(W), 0), x.send_cnt.assign(size_t(W), 0);
    x.recv_off.assign(size_t(W), 0), x.recv_cnt.assign(size_t(W), 0);
    std::vector<int32_t> idx;
    for (int p = 0; p < W; ++p) {
        x.send_off[size_t(p)] = int64_t(idx.size()) * row;
        for (int32_t g : h.send[size_t(p)]) idx.push_back(int32_t(g - lo));
        x.send_cnt[size_t(p)] = int64_t(h.send[size_t(p)].size()) * row;
    }
    int64_t off = 0;
    for (int p = 0; p < W; ++p) {
        x.recv_off[size_t(p)] = off * row;
        x.recv_cnt[size_t(p)] = h.recv_count[size_t(p)] * row;
        off += h.recv_count[size_t(p)];
    }
    x.n_send = int64_t(idx.size());
    x.n_recv = off;
    if (idx.empty()) idx.push_back(0);
    x.send_idx = upload(idx.data(), idx.size() * sizeof(int32_t));
}

// Halo exchange of K|V rows (2C wide): pack the own rows every peer needs from src (row stride lds)
// into xsend_, grouped send/recv; the received rows (ascending global id = peer order) land in
// dst rows [0, n_recv) (stride ldd) directly when `direct` (contiguous 2C rows), else via xrecv_.
template <class T>
void Engine<T>::exchange(Xchg& x, const T* src, int64_t lds, T* dst, int64_t ldd, bool direct, cudaStream_t s) {
    if (plan_.world == 1) return;
    const int64_t row = 2 * int64_t(C_);
    {
        Span sp(this, s, "halo_pack", 0, double(x.n_send) * row * 2 * sizeof(T));
        k::copy_rows<T>(xsend_, row, nullptr, src, lds, x.send_idx.template as<int32_t>(), x.n_send, row, s);
    }
    T* recv = direct ? dst : xrecv_;
    {
        Span sp(this, s, "halo_exchange", 0, double(x.n_send + x.n_recv) * row * sizeof(T));
        comm_->exchange(xsend_, x.send_off, x.send_cnt, recv, x.recv_off, x.recv_cnt, int(sizeof(T)), s);
    }
    if (!direct) {
        Span sp(this, s, "halo_unpack", 0, double(x.n_recv) * row * 2 * sizeof(T));
        k::copy_rows<T>(dst, ldd, nullptr, xrecv_, row, nullptr, x.n_recv, row, s);
    }
}

// Encoder split: the encoder's output rows (src, [El, C], rows [e_lo, e_hi)) to their processor owners
// (dst, [Hl, C], rows [h_lo, h_hi)). Both sides are contiguous row ranges per peer, so the rows go
// straight from src and into dst, without packing.
template <class T>
void Engine<T>::enc_redistribute(const T* src, T* dst, cudaStream_t s) {
    double rows = double(emove_.self_rows);
    for (int64_t n : emove_.send_cnt) rows += double(n) / double(C_);
    for (int64_t n : emove_.recv_cnt) rows += double(n) / double(C_);
    Span sp(this, s, "enc_redistribute", 0, rows * double(C_) * sizeof(T));
    if (emove_.self_rows > 0)
        VB_CUDA(cudaMemcpyAsync(dst + emove_.self_dst * C_, src + emove_.self_src * C_,
                                size_t(emove_.self_rows * C_) * sizeof(T), cudaMemcpyDeviceToDevice, s));
    comm_->exchange(src, emove_.send_off, emove_.send_cnt, dst, emove_.recv_off, emove_.recv_cnt, int(sizeof(T)), s);
}

template <class T>
T* Engine<T>::act(size_t elems) {
    acts_.emplace_back(align_up(std::max<size_t>(1, elems) * sizeof(T), 256));
    act_bytes_ += acts_.back().bytes();
    return acts_.back().template as<T>();
}

template <class T>
float* Engine<T>::actf(size_t elems) {
    acts_.emplace_back(align_up(std::max<size_t>(1, elems) * sizeof(float), 256));
    act_bytes_ += acts_.back().bytes();
    return acts_.back().template as<float>();
}

template <class T>
Engine<T>::Engine(const std::string& path, const Options& o) : opts_(o) {
    dev_ = o.cuda_device;
    LoadTimer lt;
    SafeTensorsFile file(path);
    if (file.metadata("varda_format") != "1")
        fail(kFormat, path + ": unsupported varda_format " + file.metadata("varda_format"));
    cfg_ = parse_config(file.metadata("config"));
    validate_model_file(file, cfg_);  // format errors surface before any device call
    VB_CUDA(cudaSetDevice(dev_));
    file.prefetch();
    const Config& c = cfg_;
    C_ = c.num_channels, heads_ = c.num_heads, hd_ = c.head_dim, mlp_ = c.mlp_hidden;
    n_proc_ = c.num_processor_layers, T_in_ = c.n_input_steps, T_out_ = c.n_output_steps;
    V_in_ = c.n_input_vars, V_out_ = c.n_output_vars, V_dec_ = c.dec_out_features();
    A_node_ = c.node_attr_dim, G_ = c.n_data_nodes, H_ = c.n_hidden_nodes;
    eps_ = c.layer_norm_eps, gelu_tanh_ = c.gelu_tanh;
    F_ = c.src_features();
    ldF_ = int64_t(align_up(size_t(F_), 8));
    ldA_ = int64_t(align_up(size_t(A_node_), 8));
    ldVo_ = int64_t(align_up(size_t(V_dec_), 8));
    if (C_ % 128 || C_ > 2048) fail(kUnsupported, "num_channels must be a multiple of 128, <= 2048");
    if (hd_ % 4 || hd_ > 256) fail(kUnsupported, "head_dim must be a multiple of 4, <= 256");
    if (mlp_ % 8) fail(kUnsupported, "mlp_hidden must be a multiple of 8");
    if (c.edge_attr_dim < 1 || c.edge_attr_dim > 3) fail(kUnsupported, "edge_attr_dim must be 1..3");
    if (n_proc_ < 1) fail(kUnsupported, "needs at least one processor block");
    const bool fp16 = !std::is_same<T, float>::value;
    use_tc_ = fp16 && opts_.gemm == 0 && env_int("VB_GEMM_SIMT", 0) == 0;
    VB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    gemm_sched_.alloc(4 * sizeof(unsigned));
    VB_CUDA(cudaMemset(gemm_sched_.get(), 0, 4 * sizeof(unsigned)));
    if (env_int("VB_GEMM_SCHED", 1) != 0) sched_ = gemm_sched_.as<unsigned>();
    if (env_int("VB_ATT_SCHED", 1) != 0) att_sched_ = gemm_sched_.as<unsigned>() + 2;

    // ---- normaliser, residual, bounding
    const TensorView& mul = file.take("norm.mul", DType::F32, {c.n_data_vars});
    const TensorView& add = file.take("norm.add", DType::F32, {c.n_data_vars});
    std::vector<float> mi, ai, mo, ao;
    for (int i : c.norm_input) mi.push_back(mul.as<float>()[i]), ai.push_back(add.as<float>()[i]);
    for (int i : c.norm_output) mo.push_back(mul.as<float>()[i]), ao.push_back(add.as<float>()[i]);
    mul_in_ = upload(mi.data(), mi.size() * 4);
    add_in_ = upload(ai.data(), ai.size() * 4);
    mul_out_ = upload(mo.data(), mo.size() * 4);
    add_out_ = upload(ao.data(), ao.size() * 4);
    std::vector<int> rs(size_t(V_out_), -1);
    for (size_t k2 = 0; k2 < c.residual_output.size(); ++k2) rs[size_t(c.residual_output[k2])] = c.residual_input[k2];
    res_src_ = upload(rs.data(), rs.size() * 4);
    std::vector<k::BoundDev> bd;
    std::vector<int> bidx;
    for (const Bounding& b : c.bounding) {
        k::BoundDev d;
        d.type = b.type == "relu" ? 0 : b.type == "hardtanh" ? 1 : 2;
        d.n = int(b.index.size());
        d.idx_off = int(bidx.size());
        bidx.insert(bidx.end(), b.index.begin(), b.index.end());
        d.tot_off = int(bidx.size());
        d.n_tot = int(b.total_index.size());
        bidx.insert(bidx.end(), b.total_index.begin(), b.total_index.end());
        d.lo = b.min, d.hi = b.max;
        for (int i : b.index)
            for (int t : b.total_index)
                if (i == t) fail(kUnsupported, "fraction bounding index overlaps its total_index");
        bd.push_back(d);
    }
    n_bounds_ = int(bd.size());
    if (bidx.empty()) bidx.push_back(0);
    if (bd.empty()) bd.push_back(k::BoundDev{});
    bounds_ = upload(bd.data(), bd.size() * sizeof(k::BoundDev));
    bidx_ = upload(bidx.data(), bidx.size() * 4);

    // ---- graphs and the destination partition (the identity on one GPU)
    {
        lt.mark("open + config");
        CsrGraph enc = read_graph(file, "enc", G_, H_);
        CsrGraph proc = read_graph(file, "proc", H_, H_);
        CsrGraph dec = read_graph(file, "dec", H_, G_);
        lt.mark("CSR build");
        plan_ = make_plan(cfg_, enc, proc, dec, opts_.world, opts_.rank, enc_split_requested());
        lt.mark("partition plan");
    }
    Hl_ = plan_.h_hi - plan_.h_lo, Gl_ = plan_.g_hi - plan_.g_lo;
    n_eh_ = int64_t(plan_.enc_halo.size()), n_ph_ = int64_t(plan_.proc.halo.size());
    n_dh_ = int64_t(plan_.dec.halo.size()), Gx_ = Gl_ + n_eh_;
    El_ = plan_.e_hi - plan_.e_lo;
    emove_.on = plan_.e_split != plan_.h_split;
    if (emove_.on) {  // the plan's row ranges as element offsets into [El, C] and [Hl, C]
        const int W = plan_.world;
        const ShardPlan::RowMove& m = plan_.enc_move;
        for (auto* v : {&emove_.send_off, &emove_.send_cnt, &emove_.recv_off, &emove_.recv_cnt}) v->assign(size_t(W), 0);
        for (int p = 0; p < W; ++p) {
            const int64_t slo = m.send_lo[size_t(p)], shi = m.send_hi[size_t(p)];
            const int64_t rlo = m.recv_lo[size_t(p)], rhi = m.recv_hi[size_t(p)];
            if (p == plan_.rank) {
                emove_.self_src = slo - plan_.e_lo, emove_.self_dst = slo - plan_.h_lo;
                emove_.self_rows = std::max<int64_t>(0, shi - slo);
                continue;
            }
            if (shi > slo) emove_.send_off[size_t(p)] = (slo - plan_.e_lo) * C_, emove_.send_cnt[size_t(p)] = (shi - slo) * C_;
            if (rhi > rlo) emove_.recv_off[size_t(p)] = (rlo - plan_.h_lo) * C_, emove_.recv_cnt[size_t(p)] = (rhi - rlo) * C_;
        }
    }
    {
        // decoder destination chunk: all own data rows in one chunk unless limited
        int64_t rows = opts_.dec_chunk_rows > 0 ? opts_.dec_chunk_rows : env_int("VB_DEC_CHUNK_ROWS", Gl_);
        rows = std::min<int64_t>(std::max<int64_t>(rows, 1), std::max<int64_t>(Gl_, 1));
        const int64_t nch = (std::max<int64_t>(Gl_, 1) + rows - 1) / rows;
        dec_rows_ = std::min<int64_t>(int64_t(align_up(size_t((Gl_ + nch - 1) / nch), 128)), std::max<int64_t>(Gl_, 1));
    }
    g_enc_ = upload_graph(plan_.enc, "enc", 0);
    lt.mark("encoder graph upload");
    g_proc_ = upload_graph(plan_.proc_g, "proc", 0);
    if (plan_.world > 1) {  // processor rows with and without a remote (halo) source
        std::vector<int32_t> inner, outer;
        const CsrGraph& pg = plan_.proc_g;
        for (int64_t r = 0; r < pg.n_dst; ++r) {
            bool remote = false;
            for (int32_t e = pg.row_ptr[size_t(r)]; e < pg.row_ptr[size_t(r + 1)] && !remote; ++e)
                remote = pg.src[size_t(e)] >= Hl_;
            (remote ? outer : inner).push_back(int32_t(r));
        }
        if (int64_t(inner.size() + outer.size()) != Hl_) fail(kInternal, "processor row split");
        n_inner_ = int64_t(inner.size()), n_outer_ = int64_t(outer.size());
        proc_inner_ = upload(inner.data(), std::max<size_t>(1, inner.size()) * sizeof(int32_t));
        proc_outer_ = upload(outer.data(), std::max<size_t>(1, outer.size()) * sizeof(int32_t));
        if (g_proc_.tc) {
            const TcPlan tp = make_tc_tiles(pg, kTcAlignRows);  // the same tiles upload_graph built
            std::vector<TcTile> in_t, out_t;
            for (const TcTile& t : tp.tiles) {
                bool remote = false;
                for (int i = 0; i < t.nsrc && !remote; ++i) remote = tp.srcs[size_t(t.src_off + i)] >= Hl_;
                (remote ? out_t : in_t).push_back(t);
            }
            n_tc_inner_ = int(in_t.size()), n_tc_tiles_ = int(tp.tiles.size());
            in_t.insert(in_t.end(), out_t.begin(), out_t.end());
            proc_tc_tiles_ = upload(in_t.data(), std::max<size_t>(1, in_t.size()) * sizeof(TcTile));
            std::vector<int32_t> hin, hout;
            for (int32_t r : tp.heavy)
                (std::binary_search(inner.begin(), inner.end(), r) ? hin : hout).push_back(r);
            n_heavy_inner_ = int64_t(hin.size()), n_heavy_outer_ = int64_t(hout.size());
            proc_heavy_inner_ = upload(hin.data(), std::max<size_t>(1, hin.size()) * sizeof(int32_t));
            proc_heavy_outer_ = upload(hout.data(), std::max<size_t>(1, hout.size()) * sizeof(int32_t));
        }
    }
    // pipelined host I/O: decoder chunks of ~Gl / VB_IO_CHUNKS rows (the memory cap's chunks if set),
    // input chunks of ~Gl / (2 VB_IO_CHUNKS) own rows; the decoder tiles respect the chunk boundaries. On C1
    // the copies (1.22 GB in at 56 GB/s, 0.54 GB out) then add ~7 ms to the 176-180 ms step instead of ~26.
    io_.on = env_int("VB_IO_PIPELINE", 1) != 0;
    if (io_.on) {
        const int64_t nio = std::max<int64_t>(1, env_int("VB_IO_CHUNKS", 8)), gl = std::max<int64_t>(Gl_, 1);
        io_.dec_rows = dec_rows_ < Gl_ ? dec_rows_
                                       : std::min<int64_t>(int64_t(align_up(size_t((gl + nio - 1) / nio), 128)), gl);
        io_.in_rows = std::min<int64_t>(int64_t(align_up(size_t((gl + 2 * nio - 1) / (2 * nio)), 128)), gl);
    }
    const int64_t dec_tile_chunk = io_.on ? io_.dec_rows : dec_rows_;
    g_dec_ = upload_graph(plan_.dec_g, "dec", dec_tile_chunk < Gl_ ? dec_tile_chunk : 0);
    lt.mark("processor + decoder graphs");
    for (CsrGraph* g : {&plan_.enc, &plan_.proc_g, &plan_.dec_g}) *g = CsrGraph{};  // host copies not needed

    // ---- node attributes: data rows [own | encoder halo], own hidden rows (and the optional grid
    // coordinates, consumed as the reference does)
    if (file.has("grid.latitudes") || file.has("grid.longitudes")) {
        file.take("grid.latitudes", DType::F64, {G_});
        file.take("grid.longitudes", DType::F64, {G_});
    }
    for (const auto& kv : file.metadata())
        if (kv.first == "cutout") fail(kUnsupported, "multi-source (cutout) grids are not supported");
    const TensorView& da = file.take("nodes.data.attr", DType::F32, {G_, A_node_});
    const TensorView& ha = file.take("nodes.hidden.attr", DType::F32, {H_, A_node_});
    {
        std::vector<float> dl(size_t(Gx_ * A_node_));
        std::memcpy(dl.data(), da.as<float>() + plan_.g_lo * A_node_, size_t(Gl_ * A_node_) * sizeof(float));
        for (int64_t i = 0; i < n_eh_; ++i)
            std::memcpy(&dl[size_t((Gl_ + i) * A_node_)], da.as<float>() + int64_t(plan_.enc_halo[size_t(i)]) * A_node_,
                        size_t(A_node_) * sizeof(float));
        d_attr_ = upload(dl.data(), dl.size() * sizeof(float));
    }
    if (plan_.world == 1) h_attr_host_.assign(ha.as<float>(), ha.as<float>() + ha.numel());
    {
        std::vector<T> hp(size_t(El_ * ldA_), T(0.0f));  // the encoder's destination rows
        for (int64_t r = 0; r < El_; ++r)
            for (int a = 0; a < A_node_; ++a)
                hp[size_t(r * ldA_ + a)] = T(ha.as<float>()[(plan_.e_lo + r) * A_node_ + a]);
        h_attr_ = upload(hp.data(), hp.size() * sizeof(T));
    }

    lt.mark("node attributes");
    // ---- weights
    {
        ParamLoader<T> pl(file, cfg_, weight_bytes_);
        enc_emb_src_ = pl.dense({"enc.emb_src"}, C_, F_);
        enc_emb_dst_ = pl.dense({"enc.emb_dst"}, C_, A_node_);
        dec_emb_dst_ = pl.dense({"dec.emb_dst"}, C_, F_);
        dec_out_norm_ = pl.affine("dec.out_norm", C_);
        dec_out_proj_ = pl.dense({"dec.out_proj"}, V_dec_, C_);
        enc_ = pl.layer("enc.block", true, C_, mlp_);
        for (int i = 0; i < n_proc_; ++i) proc_.push_back(pl.layer("proc." + std::to_string(i), false, C_, mlp_));
        dec_ = pl.layer("dec.block", true, C_, mlp_);
    }
    file.require_all_consumed();
    {
        const int lnf = use_tc_ ? env_int("VB_LN_FOLD", 1) : 0;
        fold_ = lnf != 0, fold_mlp_ = lnf >= 2;
    }
    if constexpr (std::is_same<T, __half>::value) {
        if (fold_) {
            segw_ = tc::stats_segw(C_), nseg_ = C_ / segw_;
            auto fold = [&](Dense<T>& L, const Affine& n) {
                if (!L.bias.get()) {
                    L.bias.alloc(size_t(L.out) * sizeof(T));
                    VB_CUDA(cudaMemset(L.bias.get(), 0, size_t(L.out) * sizeof(T)));
                }
                L.colsum.alloc(size_t(L.out) * sizeof(float));
                weight_bytes_ += size_t(L.out) * sizeof(float);
                k::fold_layernorm(L.weight.template as<__half>(), L.ld_in, L.out, int(L.in), n.g(), n.b(),
                                  L.bias.template as<__half>(), L.colsum.template as<float>(), stream_);
            };
            fold(enc_.proj_kv, enc_.norm_src);
            fold(enc_.proj_qx, enc_.norm_dst);
            for (AttnLayer<T>& b : proc_) fold(b.proj_qkvx, b.norm_dst);
            if (!cfg_.latent_skip) fold(dec_.proj_kv, dec_.norm_src);  // else LN(latent + skip) by add_layernorm
            fold(dec_.proj_qx, dec_.norm_dst);
            fold(dec_out_proj_, dec_out_norm_);
            if (fold_mlp_) {
                fold(enc_.ffn_up, enc_.norm_ffn);
                for (AttnLayer<T>& b : proc_) fold(b.ffn_up, b.norm_ffn);
                fold(dec_.ffn_up, dec_.norm_ffn);
            }
            VB_CUDA(cudaStreamSynchronize(stream_));
        }
    }

    lt.mark("weights");
    // ---- activations (this rank's rows)
    x_dev_ = actf(size_t(input_numel()));
    xn_ = actf(size_t(input_numel()));
    yn_ = actf(size_t(output_numel()));
    y_dev_ = actf(size_t(output_numel()));
    x_data_ = act(size_t(Gx_ * ldF_));
    dec_out_ = act(size_t(Gl_ * ldVo_));
    // hidden-row buffers: own processor rows, or the encoder's rows where it has more (encoder split)
    const int64_t Hm = std::max(Hl_, El_);
    z_enc_ = act(size_t(Hl_ * C_));
    zA_ = act(size_t(Hm * C_));
    zB_ = act(size_t(Hm * C_));
    xh_ = act(size_t(Hm * C_));
    // q|k|v|self of own rows plus the K|V of the processor halo rows; later the decoder's k|v of
    // own rows plus its halo (first the encoder's q|self)
    qkvs_ = act(size_t(std::max({(Hl_ + n_ph_) * 4 * C_, (Hl_ + n_dh_) * 2 * C_, El_ * 2 * C_})));
    sbuf_ = act(size_t(Hm * C_));
    out1_ = act(size_t(Hm * C_));
    hbuf_ = act(size_t(Hm * mlp_));
    if (fold_) {  // records of the encoder's source rows, the hidden rows or a decoder chunk
        const int64_t rows = std::max({Gx_, Hm, dec_rows_});
        stA_ = reinterpret_cast<float2*>(actf(size_t(rows * nseg_ * 2)));
        if (fold_mlp_) stB_ = reinterpret_cast<float2*>(actf(size_t(rows * nseg_ * 2)));
    }
    // Shared region: the encoder's source side ([Gx, C] embedding + [Gx, 2C] k|v), then the decoder's
    // destination chunks (6C + mlp per row). All own data rows in one chunk unless limited.
    const int64_t enc_elems = Gx_ * 3 * C_;
    const int64_t per_row = 6 * int64_t(C_) + mlp_;
    region_ = act(size_t(std::max(enc_elems, dec_rows_ * per_row)));

    // ---- halo exchanges (multi-GPU)
    if (plan_.world > 1) {
        if (!opts_.nccl_id) fail(kInvalidArgument, "sharded load needs the NCCL unique id");
        setup_exchange(xp_, plan_.proc, plan_.h_lo, 2 * int64_t(C_));
        setup_exchange(xd_, plan_.dec, plan_.h_lo, 2 * int64_t(C_));
        xsend_ = act(size_t(std::max<int64_t>(1, std::max(xp_.n_send, xd_.n_send)) * 2 * C_));
        xrecv_ = act(size_t(std::max<int64_t>(1, xp_.n_recv) * 2 * C_));
        setup_exchange(xx_, plan_.enc_x, plan_.g_lo, int64_t(T_in_) * V_in_);
        xx_send_ = actf(size_t(std::max<int64_t>(1, xx_.n_send) * T_in_ * V_in_));
        xx_recv_ = actf(size_t(std::max<int64_t>(1, xx_.n_recv) * T_in_ * V_in_));
        lt.mark("activations + exchange plans");
        comm_ = std::make_unique<Comm>(plan_.world, plan_.rank, opts_.nccl_id);
        lt.mark("NCCL communicator");
        VB_CUDA(cudaStreamCreateWithFlags(&cs_, cudaStreamNonBlocking));
        VB_CUDA(cudaEventCreateWithFlags(&ev_kv_, cudaEventDisableTiming));
        VB_CUDA(cudaEventCreateWithFlags(&ev_halo_, cudaEventDisableTiming));

    }
    VB_CUDA(cudaDeviceSynchronize());
    lt.mark("done");
}

template <class T>
Engine<T>::~Engine() {
    cudaSetDevice(dev_);
    if (stream_) cudaStreamSynchronize(stream_);
    if (graph_exec_) cudaGraphExecDestroy(graph_exec_);  // before the communicator its nodes use
    rollout_release();
    io_release();
    if (cs_) cudaStreamSynchronize(cs_), cudaStreamDestroy(cs_);
    if (ev_kv_) cudaEventDestroy(ev_kv_);
    if (ev_halo_) cudaEventDestroy(ev_halo_);
    for (cudaEvent_t e : blk_ev_)
        if (e) cudaEventDestroy(e);
    comm_.reset();
    if (stream_) cudaStreamDestroy(stream_);
}

template <class T>
void Engine<T>::use_high_priority_stream() {
    VB_CUDA(cudaSetDevice(dev_));
    int least = 0, greatest = 0;
    VB_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
    cudaStream_t s = nullptr;
    VB_CUDA(cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, greatest));
    VB_CUDA(cudaStreamSynchronize(stream_));
    VB_CUDA(cudaStreamDestroy(stream_));
    stream_ = s;
}

// ====================================================================== forward

template <class T>
void Engine<T>::linear(const Dense<T>& L, const T* x, int64_t ldx, T* y, int64_t ldy, int64_t M, cudaStream_t s,
                       int epi, const T* R, int64_t ldr, float2* st_out, const float2* st_in) {
    if (M <= 0) return;
    k::GemmArgs<T> a;
    a.A = x, a.lda = ldx, a.W = L.w(), a.ldw = L.ld_in, a.bias = L.b(), a.C = y, a.ldc = ldy;
    a.R = R, a.ldr = ldr, a.M = M, a.N = L.out, a.K = L.in, a.epi = epi, a.gelu_tanh = gelu_tanh_;
    if (fold_) {
        a.st_out = st_out;
        if (st_in) a.st_in = st_in, a.colsum = L.cs(), a.nseg_in = nseg_, a.segw_in = segw_, a.eps = eps_;
        if (bool(st_in) != bool(L.cs())) fail(kInternal, "linear: LayerNorm fold mismatch");
    }
    if constexpr (std::is_same<T, __half>::value) {
        if (use_tc_ && tc::supported(a)) {
            Span sp(this, s, "gemm_tc M=" + std::to_string(M) + " N=" + std::to_string(L.out) + " K=" +
                                 std::to_string(L.in) + " epi=" + std::to_string(epi) + (a.st_in ? " +ln" : ""),
                    2.0 * double(M) * double(L.out) * double(L.in), 0);
            tc::gemm(a, s, sched_);
            return;
        }
    }
    if (a.st_in || a.st_out) fail(kInternal, "linear: LayerNorm fusion needs the tensor-core GEMM");
    Span sp(this, s, "gemm_simt M=" + std::to_string(M) + " N=" + std::to_string(L.out) + " K=" + std::to_string(L.in) +
                         " epi=" + std::to_string(epi), 2.0 * double(M) * double(L.out) * double(L.in), 0);
    k::gemm_simt<T>(a, s);
}

template <class T>
void Engine<T>::row_stats(const T* x, int64_t rows, float2* st, cudaStream_t s) {
    if constexpr (std::is_same<T, __half>::value) {
        Span sp(this, s, "ln_stats", 0, double(rows) * (C_ * sizeof(T) + nseg_ * sizeof(float2)));
        k::row_seg_stats(x, C_, rows, C_, segw_, st, s);
    } else {
        fail(kInternal, "row_stats: fp16 only");
    }
}

template <class T>
void Engine<T>::attention(const GraphDev& g, const AttnLayer<T>& b, int64_t lo, int64_t n, const T* q, int64_t ldq,
                          const T* kk, const T* v, int64_t ldkv, const T* xr, int64_t ldxr, T* out, cudaStream_t s) {
    k::AttnArgs<T> a;
    a.row_ptr = g.rp(), a.edges = g.ed(), a.dst_lo = lo, a.n_rows = n;
    a.q = q, a.ldq = ldq, a.k = kk, a.v = v, a.ldkv = ldkv, a.xr = xr, a.ldxr = ldxr, a.out = out, a.ldo = C_;
    a.w_e = b.edge_fold.template as<float>(), a.C = C_, a.heads = heads_, a.head_dim = hd_;
    // compulsory bytes: q, x_r, out per destination, k and v per source, one 16-byte record per
    // edge, row_ptr, the [4, C] edge weights
    double edges = 0;
    if (prof_) {
        int32_t e0 = 0, e1 = 0;
        VB_CUDA(cudaMemcpy(&e0, g.rp() + lo, 4, cudaMemcpyDeviceToHost));
        VB_CUDA(cudaMemcpy(&e1, g.rp() + lo + n, 4, cudaMemcpyDeviceToHost));
        edges = double(e1 - e0);
    }
    const double bytes = double(sizeof(T)) * C_ * (3.0 * n + 2.0 * double(g.n_src)) + 16.0 * edges + 4.0 * (n + 1) +
                         16.0 * C_;
    Span sp(this, s, "attention " + g.name, 0, bytes);
    if constexpr (std::is_same<T, __half>::value) {
        if (g.tiled) {
            // tiles of rows [lo, lo + n) (tiles never straddle a decoder chunk), then the heavy rows
            const auto t0 = std::lower_bound(g.tile_row0.begin(), g.tile_row0.end(), int32_t(lo));
            const auto t1 = std::lower_bound(g.tile_row0.begin(), g.tile_row0.end(), int32_t(lo + n));
            if (g.tc) {
                k::TcArgs t;
                t.tiles = g.tiles.template as<TcTile>(), t.srcs = g.srcs.template as<int32_t>();
                t.blob = g.tblob.template as<uint8_t>();
                t.tile0 = int(t0 - g.tile_row0.begin()), t.ntiles = int(t1 - t0), t.dst_lo = lo;
                t.q = q, t.k = kk, t.v = v, t.xr = xr, t.out = out, t.ldq = ldq, t.ldkv = ldkv, t.ldxr = ldxr;
                t.ldo = C_, t.n_q_rows = n, t.n_src = g.n_src, t.w_e = a.w_e, t.C = C_, t.heads = heads_;
                t.head_dim = hd_, t.sched = att_sched_;
                k::attention_tc(t, s);
            } else {
                k::TileArgs t;
                t.tiles = g.tiles.template as<int4>(), t.srcs = g.srcs.template as<int32_t>();
                t.edges = g.tedges.template as<EdgeRec>(), t.row_ptr = g.rp(), t.dst_lo = lo;
                t.tile0 = int(t0 - g.tile_row0.begin()), t.ntiles = int(t1 - t0);
                t.q = q, t.k = kk, t.v = v, t.xr = xr, t.out = out, t.ldq = ldq, t.ldkv = ldkv, t.ldxr = ldxr;
                t.ldo = C_, t.w_e = a.w_e, t.C = C_, t.heads = heads_, t.head_dim = hd_;
                k::attention_tiled(t, 1.4426950408889634f / std::sqrt(float(hd_)), s);
            }
            const auto h0 = std::lower_bound(g.heavy_rows.begin(), g.heavy_rows.end(), int32_t(lo));
            const auto h1 = std::lower_bound(g.heavy_rows.begin(), g.heavy_rows.end(), int32_t(lo + n));
            if (h1 > h0) {
                a.rows = g.heavy.template as<int32_t>() + (h0 - g.heavy_rows.begin());
                a.n_rows = int64_t(h1 - h0);
                k::attention<T>(a, s);
            }
            return;
        }
    }
    if (g.order.get() && lo == 0 && n == g.n_dst) {  // the whole graph, in source order
        a.rows = g.order.template as<int32_t>();
        k::attention<T>(a, s);
        return;
    }
    if (g.wide) {
        // rows [lo, lo + n): the light ones on the gather kernel (row list), the wide ones by parts
        const auto l0 = std::lower_bound(g.light_rows.begin(), g.light_rows.end(), int32_t(lo));
        const auto l1 = std::lower_bound(g.light_rows.begin(), g.light_rows.end(), int32_t(lo + n));
        if (l1 > l0) {
            a.rows = g.light.template as<int32_t>() + (l0 - g.light_rows.begin());
            a.n_rows = int64_t(l1 - l0);
            k::attention<T>(a, s);
        }
        const auto w0 = std::lower_bound(g.wide_rows.begin(), g.wide_rows.end(), int32_t(lo));
        const auto w1 = std::lower_bound(g.wide_rows.begin(), g.wide_rows.end(), int32_t(lo + n));
        if (w1 > w0) {
            k::PartsArgs p;
            const int64_t iw0 = w0 - g.wide_rows.begin(), iw1 = w1 - g.wide_rows.begin();
            p.parts = g.parts.template as<int4>(), p.part_lo = g.part0[size_t(iw0)];
            p.n_parts = g.part0[size_t(iw1)] - p.part_lo;
            p.wide_rows = g.wide_dev.template as<int32_t>(), p.part0 = g.part0_dev.template as<int32_t>();
            p.wide_lo = iw0, p.n_wide = iw1 - iw0, p.scratch = g.scratch.template as<float>();
            a.rows = nullptr, a.n_rows = n;
            k::attention_parts<T>(a, p, s);
        }
        return;
    }
    k::attention<T>(a, s);
}

// The processor attention of the rows with no remote source (boundary false) or of the others: the
// tensor-core kernel over the interior or boundary tiles (and the heavy rows among those rows on the
// gather kernel), or the gather kernel over the row list.
template <class T>
void Engine<T>::proc_attention_part(const AttnLayer<T>& b, bool boundary, cudaStream_t s) {
    const int64_t C = C_, H = Hl_;
    const T *q = qkvs_, *kk = qkvs_ + C, *v = qkvs_ + 2 * C, *xr = qkvs_ + 3 * C;
    if constexpr (std::is_same<T, __half>::value) {
        if (g_proc_.tc) {
            const int t0 = boundary ? n_tc_inner_ : 0, t1 = boundary ? n_tc_tiles_ : n_tc_inner_;
            if (t1 > t0) {
                k::TcArgs t;
                t.tiles = proc_tc_tiles_.template as<TcTile>(), t.srcs = g_proc_.srcs.template as<int32_t>();
                t.blob = g_proc_.tblob.template as<uint8_t>();
                t.tile0 = t0, t.ntiles = t1 - t0, t.dst_lo = 0;
                t.q = q, t.k = kk, t.v = v, t.xr = xr, t.out = sbuf_, t.ldq = 4 * C, t.ldkv = 4 * C, t.ldxr = 4 * C;
                t.ldo = C, t.n_q_rows = H, t.n_src = g_proc_.n_src, t.w_e = b.edge_fold.template as<float>();
                t.C = int(C), t.heads = heads_, t.head_dim = hd_, t.sched = att_sched_;
                k::attention_tc(t, s);
            }
            attention_rows(g_proc_, b, boundary ? proc_heavy_outer_ : proc_heavy_inner_,
                           boundary ? n_heavy_outer_ : n_heavy_inner_, q, 4 * C, kk, v, 4 * C, xr, 4 * C, sbuf_, s);
            return;
        }
    }
    attention_rows(g_proc_, b, boundary ? proc_outer_ : proc_inner_, boundary ? n_outer_ : n_inner_, q, 4 * C, kk, v,
                   4 * C, xr, 4 * C, sbuf_, s);
}

// The gather attention over an explicit list of rows (local ids) of graph g.
template <class T>
void Engine<T>::attention_rows(const GraphDev& g, const AttnLayer<T>& b, const DeviceBuffer& rows, int64_t n, const T* q,
                               int64_t ldq, const T* kk, const T* v, int64_t ldkv, const T* xr, int64_t ldxr, T* out,
                               cudaStream_t s) {
    if (n <= 0) return;
    k::AttnArgs<T> a;
    a.row_ptr = g.rp(), a.edges = g.ed(), a.dst_lo = 0, a.n_rows = n, a.rows = rows.template as<int32_t>();
    a.q = q, a.ldq = ldq, a.k = kk, a.v = v, a.ldkv = ldkv, a.xr = xr, a.ldxr = ldxr, a.out = out, a.ldo = C_;
    a.w_e = b.edge_fold.template as<float>(), a.C = C_, a.heads = heads_, a.head_dim = hd_;
    k::attention<T>(a, s);
}

// Encoder source side on data rows [r0, r0 + n) of the Gx rows: assemble (the T_in input slots slot_rows
// rows apart), emb_src, LN_src (in place), [k | v]. Row-wise, so any split of the rows gives the same bits.
template <class T>
void Engine<T>::enc_source(const float* xn, int64_t slot_rows, int64_t r0, int64_t n, cudaStream_t s, HookSink* hk) {
    if (n <= 0) return;
    const int64_t G = Gx_, C = C_;
    {
        Span sp(this, s, "assemble", 0, double(n) * (T_in_ * V_in_ * 4 + A_node_ * 4 + ldF_ * sizeof(T)));
        k::assemble<T>(xn + r0 * V_in_, d_attr_.as<float>() + r0 * A_node_, T_in_, n, V_in_, A_node_,
                       x_data_ + r0 * ldF_, ldF_, s, slot_rows);
    }
    if (hk) {
        if (std::is_same<T, float>::value) {
            hk->emit("enc.x_src", x_data_, ldF_, G, F_, {G, F_});
        } else {  // the reference's x_data is fp32; the fp16 cast happens inside the Linear
            if (!hook_xsrc_.get()) hook_xsrc_.alloc(size_t(G * F_) * sizeof(float));
            k::assemble<float>(xn, d_attr_.as<float>(), T_in_, G, V_in_, A_node_, hook_xsrc_.as<float>(), F_, s);
            hk->emit("enc.x_src", hook_xsrc_.as<float>(), F_, G, F_, {G, F_});
        }
        hk->emit_host("enc.x_dst", h_attr_host_.data(), {Hl_, A_node_});
    }
    T* emb_src = region_ + r0 * C;
    T* kv_enc = region_ + G * C + r0 * 2 * C;
    float2* st = fold_ ? stA_ + r0 * nseg_ : nullptr;
    linear(enc_emb_src_, x_data_ + r0 * ldF_, ldF_, emb_src, C, n, s, k::kEpiBias, nullptr, 0, st);
    if (hk) hk->emit("enc.emb_src", emb_src, C, n, C, {n, C});
    ln_linear(enc_.norm_src, enc_.proj_kv, emb_src, st, emb_src, kv_enc, 2 * C, n, s);
}

// Encoder destination side before the attention (needs no input): emb_dst of the hidden attributes,
// LN_dst, [q | self].
template <class T>
void Engine<T>::enc_dest_pre(cudaStream_t s, HookSink* hk) {
    const int64_t H = El_, C = C_;
    T* emb_dst = zA_;
    linear(enc_emb_dst_, h_attr_.as<T>(), ldA_, emb_dst, C, H, s, k::kEpiBias, nullptr, 0, stA_);
    if (hk) hk->emit("enc.emb_dst", emb_dst, C, H, C, {H, C});
    ln_linear(enc_.norm_dst, enc_.proj_qx, emb_dst, stA_, xh_, qkvs_, 2 * C, H, s);
}

// Processor block i on this rank's hidden rows: xh_ holds LN_dst(z_in) (with fold_: stA_ holds z_in's
// records); z_out = the block's output (with fold_ its records into stA_).
template <class T>
void Engine<T>::proc_block(int i, const T* z_in, T* z_out, bool overlap, cudaStream_t s) {
    const int64_t H = Hl_, C = C_;
    const AttnLayer<T>& b = proc_[size_t(i)];
    if (fold_) linear(b.proj_qkvx, z_in, C, qkvs_, 4 * C, H, s, k::kEpiBias, nullptr, 0, nullptr, stA_);
    else linear(b.proj_qkvx, xh_, C, qkvs_, 4 * C, H, s);
    if (overlap) {
        // K|V of remote sources on the communication stream while the interior rows run
        VB_CUDA(cudaEventRecord(ev_kv_, s));
        VB_CUDA(cudaStreamWaitEvent(cs_, ev_kv_, 0));
        exchange(xp_, qkvs_ + C, 4 * C, qkvs_ + H * 4 * C + C, 4 * C, false, cs_);
        VB_CUDA(cudaEventRecord(ev_halo_, cs_));
        proc_attention_part(b, false, s);
        VB_CUDA(cudaStreamWaitEvent(s, ev_halo_, 0));
        proc_attention_part(b, true, s);
    } else {
        exchange(xp_, qkvs_ + C, 4 * C, qkvs_ + H * 4 * C + C, 4 * C, false, s);  // K|V of remote sources
        attention(g_proc_, b, 0, H, qkvs_, 4 * C, qkvs_ + C, qkvs_ + 2 * C, 4 * C, qkvs_ + 3 * C, 4 * C, sbuf_, s);
    }
    linear(b.proj_out, sbuf_, C, out1_, C, H, s, k::kEpiResidual, z_in, C, fold_mlp_ ? stB_ : nullptr);
    ln_linear(b.norm_ffn, b.ffn_up, out1_, stB_, xh_, hbuf_, mlp_, H, s, k::kEpiGelu);
    linear(b.ffn_down, hbuf_, mlp_, z_out, C, H, s, k::kEpiResidual, out1_, C, stA_);
}

// The isolated processor block (the benchmark's C2 workload): LN_dst then block `i`, `repeats` times on
// the same input, on this rank's hidden rows (sharded: with the K|V halo exchange of every run).
// z_in / z_out: host fp32 [own hidden rows, C]; a null z_in keeps the previous call's input, a null
// z_out skips the read-back. device_ms: the device time of the runs (CUDA events on the model's stream
// around them, the copies excluded). The block buffers are zA_ (input) and zB_ (output), which only a
// forward pass otherwise uses.
template <class T>
void Engine<T>::processor_block(int i, const float* z_in, float* z_out, int repeats, float* device_ms) {
    if (i < 0 || i >= n_proc_) fail(kInvalidArgument, "processor_block: no such block");
    if (repeats < 1) fail(kInvalidArgument, "processor_block: repeats must be >= 1");
    VB_CUDA(cudaSetDevice(dev_));
    cudaStream_t s = stream_;
    const int64_t H = Hl_, C = C_;
    if (!blk_stage_.get()) blk_stage_ = DeviceBuffer(size_t(std::max<int64_t>(H * C, 1)) * sizeof(float));
    float* stage = blk_stage_.as<float>();
    if (z_in) {
        VB_CUDA(cudaMemcpyAsync(stage, z_in, size_t(H * C) * sizeof(float), cudaMemcpyHostToDevice, s));
        k::convert_2d<float, T>(stage, C, zA_, C, H, C, s);
    }
    const bool overlap = plan_.world > 1 && cs_ && !prof_ && (!g_proc_.tiled || g_proc_.tc) && !g_proc_.wide &&
                         env_int("VB_SHARD_OVERLAP", 1) != 0;
    if (!blk_ev_[0]) VB_CUDA(cudaEventCreate(&blk_ev_[0])), VB_CUDA(cudaEventCreate(&blk_ev_[1]));
    VB_CUDA(cudaEventRecord(blk_ev_[0], s));
    for (int r = 0; r < repeats; ++r) {
        if (fold_) row_stats(zA_, H, stA_, s);
        else ln(zA_, proc_[size_t(i)].norm_dst, xh_, H, s);
        proc_block(i, zA_, zB_, overlap, s);
    }
    VB_CUDA(cudaEventRecord(blk_ev_[1], s));
    if (z_out) {
        k::convert_2d<T, float>(zB_, C, stage, C, H, C, s);
        VB_CUDA(cudaMemcpyAsync(z_out, stage, size_t(H * C) * sizeof(float), cudaMemcpyDeviceToHost, s));
    }
    VB_CUDA(cudaStreamSynchronize(s));
    if (device_ms) VB_CUDA(cudaEventElapsedTime(device_ms, blk_ev_[0], blk_ev_[1]));
}

// From the encoder attention to the decoder's source side ([k | v] of LN_src(latent) and its halo).
// Returns whether the decoder halo exchange is still in flight on the communication stream.
template <class T>
bool Engine<T>::middle(cudaStream_t s, HookSink* hk) {
    const int64_t G = Gx_, H = Hl_, C = C_, E = El_;
    T* kv_enc = region_ + G * C;
    T* emb_dst = zA_;
    // encoder rows [0, E): with the encoder split the output goes to zB_ (free until the second
    // processor block) and its rows then move to their processor owners' z_enc_
    T* enc_out = emove_.on ? zB_ : z_enc_;
    attention(g_enc_, enc_, 0, E, qkvs_, 2 * C, kv_enc, kv_enc + C, 2 * C, qkvs_ + C, 2 * C, sbuf_, s);
    linear(enc_.proj_out, sbuf_, C, out1_, C, E, s, k::kEpiResidual, emb_dst, C, fold_mlp_ ? stB_ : nullptr);
    ln_linear(enc_.norm_ffn, enc_.ffn_up, out1_, stB_, xh_, hbuf_, mlp_, E, s, k::kEpiGelu);
    linear(enc_.ffn_down, hbuf_, mlp_, enc_out, C, E, s, k::kEpiResidual, out1_, C, emove_.on ? nullptr : stA_);
    if (emove_.on) {
        enc_redistribute(enc_out, z_enc_, s);
        if (fold_) row_stats(z_enc_, H, stA_, s);  // the same records the epilogue would have written
    }
    if (hk) hk->emit("enc.out", z_enc_, C, H, C, {H, C});
    if (!fold_) ln(z_enc_, proc_[0].norm_dst, xh_, H, s);

    // ---- processor; xh_ holds LN_dst of the block input
    // sharded: exchange / interior-attention overlap, except under the hook or the profiler (whose
    // per-launch records stay serial) and when the processor runs the shared-memory tiled or split kernels
    const bool overlap = plan_.world > 1 && cs_ && !hk && !prof_ && (!g_proc_.tiled || g_proc_.tc) && !g_proc_.wide &&
                         env_int("VB_SHARD_OVERLAP", 1) != 0;
    T* z_in = z_enc_;
    T* latent = nullptr;
    for (int i = 0; i < n_proc_; ++i) {
        T* z_out = z_in == zA_ ? zB_ : zA_;
        proc_block(i, z_in, z_out, overlap, s);
        if (hk) hk->emit("proc." + std::to_string(i) + ".out", z_out, C, H, C, {H, C});
        if (i + 1 < n_proc_) {
            if (!fold_)  // (fold_: stA_ holds z_out's records)
                k::layernorm<T>(z_out, C, proc_[size_t(i + 1)].norm_dst.g(), proc_[size_t(i + 1)].norm_dst.b(), xh_, C,
                                H, C_, eps_, s);
        } else if (cfg_.latent_skip) {
            latent = z_in == z_enc_ ? sbuf_ : z_in;  // a dead buffer
            Span sp(this, s, "add_layernorm", 0, double(H) * C_ * 4 * sizeof(T));
            k::add_layernorm<T>(z_out, z_enc_, latent, dec_.norm_src.g(), dec_.norm_src.b(), xh_, C, H, C_, eps_, s);
        } else {
            latent = z_out;
            if (!fold_) ln(z_out, dec_.norm_src, xh_, H, s);
        }
        z_in = z_out;
    }
    if (hk) hk->emit("latent", latent, C, H, C, {H, C});

    // ---- decoder, source side: [k | v] of LN_src(latent)
    T* kv_dec = qkvs_;
    if (fold_ && !cfg_.latent_skip) linear(dec_.proj_kv, latent, C, kv_dec, 2 * C, H, s, k::kEpiBias, nullptr, 0, nullptr, stA_);
    else linear(dec_.proj_kv, xh_, C, kv_dec, 2 * C, H, s);
    if (overlap) {  // the decoder's K|V halo flies while the first chunk's destination GEMMs run
        VB_CUDA(cudaEventRecord(ev_kv_, s));
        VB_CUDA(cudaStreamWaitEvent(cs_, ev_kv_, 0));
        exchange(xd_, kv_dec, 2 * C, kv_dec + H * 2 * C, 2 * C, true, cs_);
        VB_CUDA(cudaEventRecord(ev_halo_, cs_));
        return true;
    }
    exchange(xd_, kv_dec, 2 * C, kv_dec + H * 2 * C, 2 * C, true, s);
    return false;
}

// Decoder destination rows [lo, lo + n) of the own data rows (at most dec_rows_ of them, and never
// straddling a decoder tile; the chunk buffers sit in region_), through out_proj into dec_out_.
template <class T>
void Engine<T>::dec_chunk(int64_t lo, int64_t n, cudaStream_t s, HookSink* hk, bool& halo_pending, float* h_emb,
                          float* h_bo) {
    const int64_t C = C_, R = dec_rows_;
    T* kv_dec = qkvs_;
    T* e = region_;
    T* t = e + R * C;
    T* qs = t + R * C;
    T* sb = qs + R * 2 * C;
    T* o1 = sb + R * C;
    T* h = o1 + R * C;
    linear(dec_emb_dst_, x_data_ + lo * ldF_, ldF_, e, C, n, s, k::kEpiBias, nullptr, 0, stA_);
    if (hk) hk->to_host(e, C, n, C, h_emb, lo);
    ln_linear(dec_.norm_dst, dec_.proj_qx, e, stA_, t, qs, 2 * C, n, s);
    if (halo_pending) {
        VB_CUDA(cudaStreamWaitEvent(s, ev_halo_, 0));
        halo_pending = false;
    }
    attention(g_dec_, dec_, lo, n, qs, 2 * C, kv_dec, kv_dec + C, 2 * C, qs + C, 2 * C, sb, s);
    linear(dec_.proj_out, sb, C, o1, C, n, s, k::kEpiResidual, e, C, fold_mlp_ ? stB_ : nullptr);
    ln_linear(dec_.norm_ffn, dec_.ffn_up, o1, stB_, t, h, mlp_, n, s, k::kEpiGelu);
    linear(dec_.ffn_down, h, mlp_, sb, C, n, s, k::kEpiResidual, o1, C, stA_);
    if (hk) hk->to_host(sb, C, n, C, h_bo, lo);
    ln_linear(dec_out_norm_, dec_out_proj_, sb, stA_, t, dec_out_ + lo * ldVo_, ldVo_, n, s);
}

// Output rows [lo, lo + n) of the own data rows: per step t, fp32 cast + residual + bounding into yn
// ([T_out, Gl, V_out]); xn holds the normalised input ([T_in, Gx, V_in]).
template <class T>
void Engine<T>::output_rows(const float* xn, float* yn, int64_t lo, int64_t n, cudaStream_t s, float* pre_bound) {
    k::OutputArgs o;
    o.dec = dec_out_ + lo * ldVo_, o.ld_dec = ldVo_;
    o.xn_step = xn + int64_t(cfg_.residual_step) * Gx_ * V_in_ + lo * V_in_;
    o.V_in = V_in_, o.V_out = V_out_, o.T_out = T_out_, o.G = n, o.y_slot = Gl_;
    o.res_src = res_src_.as<int>(), o.bounds = bounds_.as<k::BoundDev>(), o.n_bounds = n_bounds_;
    o.bidx = bidx_.as<int>();
    o.pre_bound = pre_bound ? pre_bound + lo * V_out_ : nullptr;
    o.y = yn + lo * V_out_;
    Span sp(this, s, "output_assemble", 0, double(n) * (ldVo_ * sizeof(T) + V_in_ * 4) + double(T_out_) * n * V_out_ * 4);
    k::output_assemble<T>(o, s);
}

template <class T>
void Engine<T>::forward(const float* xn, float* yn, cudaStream_t s, HookSink* hk) {
    const int64_t Gl = Gl_, C = C_;
    // ---- encoder: source side on all data rows (own, then the encoder's halo), destination side
    enc_source(xn, Gx_, 0, Gx_, s, hk);
    enc_dest_pre(s, hk);
    bool halo_pending = middle(s, hk);

    // ---- decoder, destination chunks of data rows
    std::vector<float> h_emb, h_bo;
    if (hk) h_emb.resize(size_t(Gl * C)), h_bo.resize(size_t(Gl * C));
    for (int64_t lo = 0; lo < Gl; lo += dec_rows_)
        dec_chunk(lo, std::min(dec_rows_, Gl - lo), s, hk, halo_pending, h_emb.data(), h_bo.data());
    if (hk) {
        hk->emit_host("dec.emb_dst", h_emb.data(), {Gl, C});
        hk->emit_host("dec.block_out", h_bo.data(), {Gl, C});
        hk->emit("dec.out", dec_out_, ldVo_, Gl, V_dec_, {Gl, int64_t(V_dec_)});
    }

    // ---- output
    if (hk && !hook_prebound_.get()) hook_prebound_.alloc(size_t(output_numel()) * sizeof(float));
    output_rows(xn, yn, 0, Gl, s, hk ? hook_prebound_.as<float>() : nullptr);
    if (hk) {
        const std::vector<int64_t> shp = {1, T_out_, 1, Gl, V_out_};
        hk->emit("out.pre_bound", hook_prebound_.as<float>(), V_out_, T_out_ * Gl, V_out_, shp);
        hk->emit("out.norm", yn, V_out_, T_out_ * Gl, V_out_, shp);
    }
}

template <class T>
void Engine<T>::prepare() {
    VB_CUDA(cudaSetDevice(dev_));
    if (ran_eager_) return;
    VB_CUDA(cudaMemsetAsync(x_dev_, 0, size_t(input_numel()) * sizeof(float), stream_));
    predict_step_device(x_dev_, y_dev_, stream_);
    VB_CUDA(cudaStreamSynchronize(stream_));
    ran_eager_ = true;
}

// Captures body(s) into an executable graph. Whatever fails inside the capture, the capture is ended,
// the partial graph destroyed and nullptr returned; the caller then runs eagerly.
template <class T>
cudaGraphExec_t Engine<T>::capture(const std::function<void(cudaStream_t)>& body, cudaStream_t s) {
    VB_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    std::string err;
    try {
        // failure-path test hook (host side): VB_DEBUG_CAPTURE_FAIL=1 fails every capture as a throwing
        // launch inside it would, so the caller's fallback to eager runs is exercised
        if (env_int("VB_DEBUG_CAPTURE_FAIL", 0) != 0) fail(kInternal, "capture failure injected (VB_DEBUG_CAPTURE_FAIL)");
        body(s);
    } catch (const std::exception& e) {
        err = e.what();
    }
    cudaGraph_t g = nullptr;
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(s, &g);
    if (err.empty() && ec != cudaSuccess) err = std::string("cudaStreamEndCapture: ") + cudaGetErrorString(ec);
    if (err.empty()) {
        const cudaError_t ei = cudaGraphInstantiate(&exec, g, 0);
        if (ei != cudaSuccess) {
            exec = nullptr;
            err = std::string("cudaGraphInstantiate: ") + cudaGetErrorString(ei);
        }
    }
    if (g) cudaGraphDestroy(g);
    if (err.empty()) return exec;
    (void)cudaGetLastError();
    std::fprintf(stderr, "varda_b200: CUDA graph capture failed (%s); running without a graph\n", err.c_str());
    return nullptr;
}

template <class T>
bool Engine<T>::capture_graph(cudaStream_t s) {
    graph_exec_ = capture([this](cudaStream_t st) { predict_step_device(x_dev_, y_dev_, st); }, s);
    return graph_exec_ != nullptr;
}

template <class T>
void Engine<T>::enqueue_predict() {
    VB_CUDA(cudaSetDevice(dev_));
    cudaStream_t s = stream_;
    if (!opts_.cuda_graph || !ran_eager_) {
        predict_step_device(x_dev_, y_dev_, s);
        ran_eager_ = true;
        return;
    }
    if (!graph_exec_ && !graph_failed_ && !capture_graph(s)) graph_failed_ = true;
    if (graph_exec_) VB_CUDA(cudaGraphLaunch(graph_exec_, s));
    else predict_step_device(x_dev_, y_dev_, s);
}

// Host x is the full (1, T_in, G, V_in) input. One GPU: one copy. Sharded: this rank's own rows (one
// contiguous range per input step); the encoder's halo rows come from their owners on the device.
template <class T>
void Engine<T>::upload_input(const float* x, cudaStream_t s) {
    if (plan_.world == 1) {
        VB_CUDA(cudaMemcpyAsync(x_dev_, x, size_t(input_numel()) * sizeof(float), cudaMemcpyHostToDevice, s));
        return;
    }
    for (int t = 0; t < T_in_; ++t)
        VB_CUDA(cudaMemcpyAsync(x_dev_ + int64_t(t) * Gx_ * V_in_, x + (int64_t(t) * G_ + plan_.g_lo) * V_in_,
                                size_t(Gl_ * V_in_) * sizeof(float), cudaMemcpyHostToDevice, s));
}

// The encoder-halo rows of x (T_in slots of V_in values each) from their owners: pack the own rows
// every peer reads, one grouped send/recv, unpack past the own rows of every slot. Every rank calls it
// (a rank with nothing to send or receive still joins the group).
template <class T>
void Engine<T>::exchange_input(float* x, cudaStream_t s) {
    if (plan_.world == 1) return;
    const int64_t slot = Gx_ * V_in_;
    {
        Span sp(this, s, "halo_pack", 0, double(xx_.n_send) * T_in_ * V_in_ * 8.0);
        k::gather_slots(xx_send_, x, T_in_, slot, xx_.send_idx.template as<int32_t>(), xx_.n_send, V_in_, s);
    }
    {
        Span sp(this, s, "halo_exchange", 0, double(xx_.n_send + xx_.n_recv) * T_in_ * V_in_ * 4.0);
        comm_->exchange(xx_send_, xx_.send_off, xx_.send_cnt, xx_recv_, xx_.recv_off, xx_.recv_cnt, int(sizeof(float)),
                        s);
    }
    {
        Span sp(this, s, "halo_unpack", 0, double(xx_.n_recv) * T_in_ * V_in_ * 8.0);
        k::scatter_slots(x, T_in_, slot, Gl_, xx_recv_, xx_.n_recv, V_in_, s);
    }
}

template <class T>
void Engine<T>::predict_step(const float* x, float* y, HookFn hook, void* user) {
    VB_CUDA(cudaSetDevice(dev_));
    cudaStream_t s = stream_;
    const int64_t in_n = input_numel(), out_n = output_numel();
    if (plan_.world > 1) {
        // y gets this rank's rows of the full (1, T_out, 1, G, V_out) output
        if (hook) fail(kUnsupported, "the activation hook is available on single-GPU models only");
        if (io_.on && opts_.cuda_graph && ran_eager_) {
            predict_pipelined(x, y);
            return;
        }
        upload_input(x, s);
        enqueue_predict();
        for (int t = 0; t < T_out_; ++t)
            VB_CUDA(cudaMemcpyAsync(y + (int64_t(t) * G_ + plan_.g_lo) * V_out_, y_dev_ + int64_t(t) * Gl_ * V_out_,
                                    size_t(Gl_ * V_out_) * sizeof(float), cudaMemcpyDeviceToHost, s));
        VB_CUDA(cudaStreamSynchronize(s));
        return;
    }
    if (io_.on && opts_.cuda_graph && ran_eager_ && !hook) {
        predict_pipelined(x, y);
        return;
    }
    VB_CUDA(cudaMemcpyAsync(x_dev_, x, size_t(in_n) * sizeof(float), cudaMemcpyHostToDevice, s));
    if (hook) {
        HookSink hk{*this, hook, user, s};
        hk.emit_host("in.x", x, {1, T_in_, G_, V_in_});
        normalise(x_dev_, xn_, s);
        hk.emit("in.x_norm", xn_, in_n, 1, in_n, {1, T_in_, 1, G_, V_in_});
        forward(xn_, yn_, s, &hk);
        denormalise(yn_, y_dev_, s);
        VB_CUDA(cudaMemcpyAsync(y, y_dev_, size_t(out_n) * sizeof(float), cudaMemcpyDeviceToHost, s));
        VB_CUDA(cudaStreamSynchronize(s));
        hk.emit_host("out.y", y, {1, T_out_, 1, G_, V_out_});
        ran_eager_ = true;
        return;
    }
    enqueue_predict();
    VB_CUDA(cudaMemcpyAsync(y, y_dev_, size_t(out_n) * sizeof(float), cudaMemcpyDeviceToHost, s));
    VB_CUDA(cudaStreamSynchronize(s));
}

// The pieces of the pipelined predict_step as graphs (eager where a capture fails), its copy stream and
// events. Runs after the first eager forward (so every lazy lookup has been done outside capture).
template <class T>
void Engine<T>::io_setup() {
    cudaStream_t s = stream_;
    VB_CUDA(cudaStreamCreateWithFlags(&io_.cio, cudaStreamNonBlocking));
    VB_CUDA(cudaEventCreateWithFlags(&io_.start, cudaEventDisableTiming));
    const int64_t n_in = (Gl_ + io_.in_rows - 1) / io_.in_rows, n_dec = (Gl_ + io_.dec_rows - 1) / io_.dec_rows;
    io_.in_done.assign(size_t(n_in), nullptr);
    io_.out_done.assign(size_t(n_dec), nullptr);
    for (cudaEvent_t& e : io_.in_done) VB_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    for (cudaEvent_t& e : io_.out_done) VB_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    // normalise + encoder source side of rows [r0, r0 + n) of the Gx rows
    auto src_rows = [this](int64_t r0, int64_t n, cudaStream_t st) {
        if (n <= 0) return;
        for (int t = 0; t < T_in_; ++t) {
            const int64_t off = (int64_t(t) * Gx_ + r0) * V_in_;
            k::normalise(x_dev_ + off, mul_in_.as<float>(), add_in_.as<float>(), xn_ + off, n * V_in_, V_in_, st);
        }
        enc_source(xn_, Gx_, r0, n, st, nullptr);
    };
    io_.pre.body = [this](cudaStream_t st) { enc_dest_pre(st, nullptr); };
    for (int64_t c = 0; c < n_in; ++c) {
        const int64_t r0 = c * io_.in_rows, n = std::min(io_.in_rows, Gl_ - r0);
        io_.src.push_back(IoSeg{[src_rows, r0, n](cudaStream_t st) { src_rows(r0, n, st); }, nullptr});
    }
    if (plan_.world > 1)  // the encoder's halo rows from their owners, then their source side
        io_.halo.body = [this, src_rows](cudaStream_t st) {
            exchange_input(x_dev_, st);
            src_rows(Gl_, n_eh_, st);
        };
    io_.mid.body = [this](cudaStream_t st) {
        if (middle(st, nullptr)) VB_CUDA(cudaStreamWaitEvent(st, ev_halo_, 0));  // the decoder halo has landed
    };
    for (int64_t d = 0; d < n_dec; ++d) {
        const int64_t lo = d * io_.dec_rows, n = std::min(io_.dec_rows, Gl_ - lo);
        io_.dec.push_back(IoSeg{[this, lo, n](cudaStream_t st) {
                                    bool pending = false;
                                    dec_chunk(lo, n, st, nullptr, pending, nullptr, nullptr);
                                    output_rows(xn_, yn_, lo, n, st, nullptr);
                                    for (int t = 0; t < T_out_; ++t) {
                                        const int64_t off = (int64_t(t) * Gl_ + lo) * V_out_;
                                        k::denormalise(yn_ + off, add_out_.as<float>(), mul_out_.as<float>(),
                                                       y_dev_ + off, n * V_out_, V_out_, st);
                                    }
                                },
                                nullptr});
    }
    // every rank captures the same pieces in the same order (the halo and mid pieces hold NCCL calls)
    auto cap = [&](IoSeg& g) {
        if (g.body) g.graph = capture(g.body, s);
    };
    cap(io_.pre);
    for (IoSeg& g : io_.src) cap(g);
    cap(io_.halo);
    cap(io_.mid);
    for (IoSeg& g : io_.dec) cap(g);
    io_.ready = true;
}

template <class T>
void Engine<T>::io_release() {
    if (io_.cio) cudaStreamSynchronize(io_.cio), cudaStreamDestroy(io_.cio);
    IoSeg* one[3] = {&io_.pre, &io_.halo, &io_.mid};
    for (IoSeg* g : one)
        if (g->graph) cudaGraphExecDestroy(g->graph);
    for (IoSeg& g : io_.src)
        if (g.graph) cudaGraphExecDestroy(g.graph);
    for (IoSeg& g : io_.dec)
        if (g.graph) cudaGraphExecDestroy(g.graph);
    for (cudaEvent_t e : io_.in_done)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : io_.out_done)
        if (e) cudaEventDestroy(e);
    if (io_.start) cudaEventDestroy(io_.start);
    io_ = IoPipe{};
}

// predict_step through host buffers with the copies overlapped: x's rows in chunks on cio_ (each
// input step's rows of a chunk, T_in copies), the encoder's destination side (which needs no input)
// first, then each chunk's normalise + source side as soon as it has landed, the rest of the encoder and
// the processor, then the decoder chunk by chunk with each chunk's output rows copied back on cio_ while
// the next one runs. The same arithmetic as the one-graph device path, row for row, so the same bits.
template <class T>
void Engine<T>::predict_pipelined(const float* x, float* y) {
    cudaStream_t s = stream_;
    if (!io_.ready) io_setup();
    // host rows of this rank: data rows [g_lo, g_hi) of every step
    VB_CUDA(cudaEventRecord(io_.start, s));  // x_dev_ / y_dev_ are free once the work before this call is done
    VB_CUDA(cudaStreamWaitEvent(io_.cio, io_.start, 0));
    for (size_t c = 0; c < io_.in_done.size(); ++c) {
        const int64_t r0 = int64_t(c) * io_.in_rows, n = std::min(io_.in_rows, Gl_ - r0);
        for (int t = 0; t < T_in_; ++t)
            VB_CUDA(cudaMemcpyAsync(x_dev_ + (int64_t(t) * Gx_ + r0) * V_in_, x + (int64_t(t) * G_ + plan_.g_lo + r0) * V_in_,
                                    size_t(n * V_in_) * sizeof(float), cudaMemcpyHostToDevice, io_.cio));
        VB_CUDA(cudaEventRecord(io_.in_done[c], io_.cio));
    }
    io_run(io_.pre, s);
    for (size_t c = 0; c < io_.in_done.size(); ++c) {
        VB_CUDA(cudaStreamWaitEvent(s, io_.in_done[c], 0));
        io_run(io_.src[c], s);
    }
    io_run(io_.halo, s);
    io_run(io_.mid, s);
    for (size_t d = 0; d < io_.out_done.size(); ++d) {
        const int64_t lo = int64_t(d) * io_.dec_rows, n = std::min(io_.dec_rows, Gl_ - lo);
        io_run(io_.dec[d], s);
        VB_CUDA(cudaEventRecord(io_.out_done[d], s));
        VB_CUDA(cudaStreamWaitEvent(io_.cio, io_.out_done[d], 0));
        for (int t = 0; t < T_out_; ++t)
            VB_CUDA(cudaMemcpyAsync(y + (int64_t(t) * G_ + plan_.g_lo + lo) * V_out_, y_dev_ + (int64_t(t) * Gl_ + lo) * V_out_,
                                    size_t(n * V_out_) * sizeof(float), cudaMemcpyDeviceToHost, io_.cio));
    }
    VB_CUDA(cudaStreamSynchronize(io_.cio));
    VB_CUDA(cudaStreamSynchronize(s));
}

// ====================================================================== rollout

// The state update of the reference's rollout (varda::StateUpdate::from_config / make,
// rollout.cpp:28-68): every input channel is exactly one of prognostic (fed back from the
// output), dynamic forcing (replayed) or constant.
template <class T>
void Engine<T>::rollout_setup() {
    if (ro_.ready) return;
    if (!cfg_.has_forcings)
        fail(kUnsupported, "rollout: the model config has no `forcings` section (dynamic/constant forcing names "
                           "and input indices)");
    if (T_out_ != 1) fail(kUnsupported, "rollout: only models with one output step are supported");
    if (cfg_.residual_input.size() != cfg_.residual_output.size())
        fail(kFormat, "rollout: residual_input and residual_output differ in length");
    ro_.F = int(cfg_.forcing_dynamic_index.size());
    ro_.kind.assign(size_t(V_in_), int8_t(-1));
    std::vector<int> src(size_t(V_in_), -1);
    auto claim = [&](int c, int k, int from, const char* what) {
        if (c < 0 || c >= V_in_) fail(kFormat, std::string("rollout: ") + what + " index out of range");
        if (ro_.kind[size_t(c)] >= 0)
            fail(kFormat, "rollout: input channel " + std::to_string(c) + " is listed twice (" + what + ")");
        ro_.kind[size_t(c)] = int8_t(k);
        src[size_t(c)] = from;
    };
    for (size_t i = 0; i < cfg_.residual_input.size(); ++i) {
        if (cfg_.residual_output[i] < 0 || cfg_.residual_output[i] >= V_out_)
            fail(kFormat, "rollout: residual_output index out of range");
        claim(cfg_.residual_input[i], 1, cfg_.residual_output[i], "prognostic");
    }
    for (int k = 0; k < ro_.F; ++k) claim(cfg_.forcing_dynamic_index[size_t(k)], 2, k, "dynamic forcing");
    for (int c : cfg_.forcing_constant_index) claim(c, 0, -1, "constant forcing");
    for (int c = 0; c < V_in_; ++c)
        if (ro_.kind[size_t(c)] < 0)
            fail(kFormat, "rollout: input channel " + std::to_string(c) +
                              " is neither prognostic, dynamic forcing nor constant: it cannot be rolled out");

    prepare();  // one eager forward before any capture
    const int64_t f_n = std::max<int64_t>(1, Gl_ * ro_.F), y_n = Gl_ * V_out_;
    ro_.d_kind.alloc(size_t(V_in_));
    ro_.d_src.alloc(size_t(V_in_) * sizeof(int));
    VB_CUDA(cudaMemcpy(ro_.d_src.get(), src.data(), size_t(V_in_) * sizeof(int), cudaMemcpyHostToDevice));
    for (int p = 0; p < 2; ++p) {
        ro_.f[p].alloc(size_t(f_n) * sizeof(float));
        VB_CUDA(cudaMemset(ro_.f[p].get(), 0, size_t(f_n) * sizeof(float)));
        ro_.y[p].alloc(size_t(std::max<int64_t>(1, y_n)) * sizeof(float));
        VB_CUDA(cudaMallocHost(&ro_.hy[p], size_t(std::max<int64_t>(1, y_n)) * sizeof(float)));
        VB_CUDA(cudaMallocHost(&ro_.hf[p], size_t(f_n) * sizeof(float)));
        VB_CUDA(cudaEventCreateWithFlags(&ro_.up[p], cudaEventDisableTiming));
        VB_CUDA(cudaEventCreateWithFlags(&ro_.down[p], cudaEventDisableTiming));
    }
    VB_CUDA(cudaStreamCreateWithFlags(&ro_.d2h, cudaStreamNonBlocking));
    VB_CUDA(cudaStreamCreateWithFlags(&ro_.h2d, cudaStreamNonBlocking));
    ro_.ready = true;
}

template <class T>
void Engine<T>::rollout_release() {
    for (auto& gp : ro_.graph)
        for (auto& g : gp)
            if (g) cudaGraphExecDestroy(g);
    cudaStream_t streams[2] = {ro_.d2h, ro_.h2d};
    for (cudaStream_t st : streams) {
        if (!st) continue;
        cudaStreamSynchronize(st);
        cudaStreamDestroy(st);
    }
    for (int p = 0; p < 2; ++p) {
        if (ro_.hy[p]) cudaFreeHost(ro_.hy[p]);
        if (ro_.hf[p]) cudaFreeHost(ro_.hf[p]);
        if (ro_.up[p]) cudaEventDestroy(ro_.up[p]);
        if (ro_.down[p]) cudaEventDestroy(ro_.down[p]);
    }
    for (cudaEvent_t e : ro_.beg) cudaEventDestroy(e);
    for (cudaEvent_t e : ro_.end) cudaEventDestroy(e);
    ro_ = Roll{};
}

// One rollout step on s: (sharded: the halo rows of every window slot from their owners) normalise
// the window -> forward -> denormalise into y[p]; with the update, the state update of this rank's
// own rows of the window in place.
template <class T>
void Engine<T>::rollout_body(int p, bool update, cudaStream_t s) {
    float* y = ro_.y[p].template as<float>();
    predict_step_device(x_dev_, y, s);
    if (!update) return;
    k::rollout_update(x_dev_, T_in_, Gl_, V_in_, y, nullptr, Gl_, V_out_, ro_.f[p].template as<float>(), ro_.F,
                      ro_.d_kind.template as<int8_t>(), ro_.d_src.template as<int>(), s, Gx_ * int64_t(V_in_));
}

// The device loop: step s (parity p = s % 2) replays graph[p] on the model's stream; its output y[p]
// goes to pinned host memory on the D2H stream and is delivered (copied into y, the callback) while
// step s + 1 runs; the forcing of step s + 1 is gathered into pinned memory and uploaded on the H2D
// stream while step s runs. Same order of operations as the reference's host loop (Rollout::run,
// rollout.cpp:116-155): predict, then (unless last) the update with forcing s.
template <class T>
void Engine<T>::rollout(const float* x0, int n, const float* forcings, float* y, bool constants_oldest, StepFn cb,
                        void* user, float* step_ms) {
    VB_CUDA(cudaSetDevice(dev_));
    if (!x0 || n < 1) fail(kInvalidArgument, "rollout: need x0 and n_steps >= 1");
    rollout_setup();
    if (n > 1 && ro_.F > 0 && !forcings) fail(kInvalidArgument, "rollout: forcings missing");
    cudaStream_t s = stream_;
    if (ro_.oldest != int(constants_oldest)) {
        std::vector<int8_t> kd = ro_.kind;
        for (auto& k : kd)
            if (k == 0 && constants_oldest) k = 3;
        VB_CUDA(cudaMemcpy(ro_.d_kind.get(), kd.data(), kd.size(), cudaMemcpyHostToDevice));
        ro_.oldest = int(constants_oldest);
    }
    for (int i = int(ro_.beg.size()); i < n; ++i) {
        cudaEvent_t a, b;
        VB_CUDA(cudaEventCreate(&a));
        VB_CUDA(cudaEventCreate(&b));
        ro_.beg.push_back(a), ro_.end.push_back(b);
    }
    const bool graphs = opts_.cuda_graph && !ro_.graph_failed;
    if (graphs && !ro_.graph[0][0]) {
        for (int p = 0; p < 2 && !ro_.graph_failed; ++p)
            for (int u = 0; u < 2 && !ro_.graph_failed; ++u) {
                ro_.graph[p][u] = capture([&](cudaStream_t st) { rollout_body(p, u == 1, st); }, s);
                if (!ro_.graph[p][u]) ro_.graph_failed = true;
            }
        for (auto& gp : ro_.graph)
            for (auto& g : gp)
                if (g) VB_CUDA(cudaGraphUpload(g, s));
    }
    const int F = ro_.F;
    const int64_t y_n = Gl_ * V_out_;
    auto produce_forcing = [&](int st) {  // forcing written after step st, into f[st % 2]
        const int b = st & 1;
        const float* fs = forcings + int64_t(st) * G_ * F;
        std::memcpy(ro_.hf[b], fs + plan_.g_lo * F, size_t(Gl_ * F) * sizeof(float));
        if (st >= 2) VB_CUDA(cudaStreamWaitEvent(ro_.h2d, ro_.end[size_t(st - 2)], 0));  // step st-2 read f[b]
        VB_CUDA(cudaMemcpyAsync(ro_.f[b].get(), ro_.hf[b], size_t(Gl_ * F) * sizeof(float), cudaMemcpyHostToDevice,
                                ro_.h2d));
        VB_CUDA(cudaEventRecord(ro_.up[b], ro_.h2d));
    };
    auto deliver = [&](int st) {
        const int b = st & 1;
        VB_CUDA(cudaEventSynchronize(ro_.down[b]));
        if (y) std::memcpy(y + (int64_t(st) * G_ + plan_.g_lo) * V_out_, ro_.hy[b], size_t(y_n) * sizeof(float));
        if (cb) cb(st, ro_.hy[b], Gl_, user);
    };

    VB_CUDA(cudaStreamSynchronize(s));
    VB_CUDA(cudaStreamSynchronize(ro_.d2h));
    VB_CUDA(cudaStreamSynchronize(ro_.h2d));
    upload_input(x0, s);
    const bool feed = F > 0 && n > 1;
    if (feed) produce_forcing(0);
    for (int st = 0; st < n; ++st) {
        const int p = st & 1;
        const bool update = st + 1 < n;  // no update after the last step
        if (update && feed) VB_CUDA(cudaStreamWaitEvent(s, ro_.up[p], 0));  // forcing st on the device
        if (st >= 2) VB_CUDA(cudaStreamWaitEvent(s, ro_.down[p], 0));       // y[p] of step st-2 copied out
        VB_CUDA(cudaEventRecord(ro_.beg[size_t(st)], s));
        if (graphs && !ro_.graph_failed) VB_CUDA(cudaGraphLaunch(ro_.graph[p][update ? 1 : 0], s));
        else rollout_body(p, update, s);
        VB_CUDA(cudaEventRecord(ro_.end[size_t(st)], s));
        VB_CUDA(cudaStreamWaitEvent(ro_.d2h, ro_.end[size_t(st)], 0));
        VB_CUDA(cudaMemcpyAsync(ro_.hy[p], ro_.y[p].get(), size_t(y_n) * sizeof(float), cudaMemcpyDeviceToHost,
                                ro_.d2h));
        VB_CUDA(cudaEventRecord(ro_.down[p], ro_.d2h));
        if (feed && st + 1 < n - 1) {
            // pinned hf[1-p] last fed the upload of forcing st-1; wait for that copy
            if (st >= 1) VB_CUDA(cudaEventSynchronize(ro_.up[1 - p]));
            produce_forcing(st + 1);
        }
        if (st >= 1) deliver(st - 1);
    }
    deliver(n - 1);
    VB_CUDA(cudaStreamSynchronize(s));
    VB_CUDA(cudaStreamSynchronize(ro_.h2d));
    if (step_ms)
        for (int st = 0; st < n; ++st)
            VB_CUDA(cudaEventElapsedTime(&step_ms[st], ro_.beg[size_t(st)], ro_.end[size_t(st)]));
    ran_eager_ = true;
}

template <class T>
std::string Engine<T>::profile_forward() {
    return profiled([&] {
        normalise(x_dev_, xn_, stream_);
        forward(xn_, yn_, stream_, nullptr);
    });
}

template <class T>
std::string Engine<T>::profile_block(int block) {
    return profiled([&] { processor_block(block, nullptr, nullptr, 1, nullptr); });
}

// Runs body() eagerly with an event pair around every launch; the records as a JSON array.
template <class T>
template <class F>
std::string Engine<T>::profiled(F body) {
    VB_CUDA(cudaSetDevice(dev_));
    std::vector<ProfRec> recs;
    prof_ = &recs;
    std::string out = "[";
    try {
        body();
        VB_CUDA(cudaStreamSynchronize(stream_));
    } catch (...) {
        prof_ = nullptr;
        throw;
    }
    prof_ = nullptr;
    for (size_t i = 0; i < recs.size(); ++i) {
        float ms = 0;
        VB_CUDA(cudaEventElapsedTime(&ms, recs[i].a, recs[i].b));
        char buf[512];
        std::snprintf(buf, sizeof buf, "%s{\"name\": \"%s\", \"ms\": %.6f, \"flop\": %.6g, \"bytes\": %.6g}", i ? ", " : "",
                      recs[i].name.c_str(), double(ms), recs[i].flop, recs[i].bytes);
        out += buf;
        cudaEventDestroy(recs[i].a);
        cudaEventDestroy(recs[i].b);
    }
    return out + "]";
}

template class Engine<float>;
template class Engine<__half>;

std::atomic<int64_t>& launch_counter() {
    static std::atomic<int64_t> n{0};
    return n;
}

std::unique_ptr<Model> load_model(const std::string& path, const Options& o) {
    if (o.precision == 0) return std::make_unique<Engine<float>>(path, o);
    return std::make_unique<Engine<__half>>(path, o);
}

}  // namespace vb
