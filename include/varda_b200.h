/* libvarda_b200 — the C ABI of the B200-native GraphTransformer backend.
 *
 * Drop-in replacement for the CUDA backend of varda.cpp (frazane/varda.cpp). Each entry point names
 * the reference interface it replaces (file:line in the reference project). Plain pointers and sizes
 * only; no C++ or torch types cross this boundary; no exception crosses it: every function returns
 * a status (VB_OK = 0, else an error class below) and vb_last_error() gives the message of the
 * calling thread's last failure.
 *
 * Ownership: the caller owns x and y (host or device buffers it passes in). The library owns every
 * device weight, graph and activation buffer of a model; they are allocated by vb_load and freed by
 * vb_free. After vb_prepare, the *_device entry points and vb_enqueue_predict only enqueue work on
 * the given stream (no allocation, no synchronisation), so a caller may capture them in its own CUDA
 * graph. At most one forward pass may be in flight per model.
 */
#ifndef VARDA_B200_H
#define VARDA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status / error classes */
#define VB_OK 0
#define VB_ERR_INVALID_ARGUMENT 1
#define VB_ERR_FORMAT 2      /* model file or config: missing/unconsumed tensor, bad shape, unknown kind */
#define VB_ERR_CUDA 3
#define VB_ERR_UNSUPPORTED 4
#define VB_ERR_INTERNAL 5
#define VB_ERR_TIMEOUT 6     /* a bounded device-side wait gave up */

#define VB_PRECISION_FP32 0
#define VB_PRECISION_FP16 1

typedef struct vb_model vb_model;

/* varda::Options (src/varda/varda.h:21-27). device is always CUDA here; num_threads is accepted
 * and ignored (it configures the reference's CPU backend). */
typedef struct {
    int precision;      /* VB_PRECISION_FP32 | VB_PRECISION_FP16 */
    int cuda_device;
    int cuda_graph;     /* nonzero: capture the forward pass once, replay afterwards */
    int num_threads;
} vb_options;

/* varda::ActivationHook (src/varda/varda.h:31-32): every contract activation once per predict_step,
 * host fp32, contiguous, row-major with `shape` (ndim entries); valid only during the call. */
typedef void (*vb_hook_fn)(const char* key, const float* data, const int64_t* shape, int ndim, void* user);

/* Message of the calling thread's last failed call ("" if none). */
const char* vb_last_error(void);

/* varda::Model::load (src/varda/varda.h:39, model.cpp:23-78) + make_cuda_backend (backend.h:25-26):
 * maps the safetensors file, parses and checks the config, uploads weights and graphs, allocates
 * every activation buffer. Strict: fails unless every tensor of the file is consumed. */
int vb_load(const char* path, const vb_options* opts, vb_model** out);

/* Multi-GPU load: one process per GPU (rank of world), the graph partitioned by destination node.
 * nccl_id: the 128-byte ncclUniqueId made by vb_nccl_unique_id on one rank and shared by the
 * caller. No reference counterpart (the reference runs one GPU). */
int vb_load_sharded(const char* path, const vb_options* opts, int rank, int world, const void* nccl_id,
                    vb_model** out);
int vb_nccl_unique_id(void* out128);

/* delete the Model / Backend (the reference's destructors). */
void vb_free(vb_model* m);

/* varda::Model::predict_step (src/varda/varda.h:50, backend.h:16): host x (1, T_in, G, V_in) fp32 in
 * physical units -> host y (1, T_out, 1, G, V_out). hook may be NULL. On a sharded model every rank
 * passes the full x and writes only its own data rows of y (vb_data_range). A bounded device-side wait
 * that gave up in the step (GEMM or attention) makes it return VB_ERR_TIMEOUT, as vb_rollout does. */
int vb_predict_step(vb_model* m, const float* x, float* y, vb_hook_fn hook, void* user);

/* Autoregressive rollout with replayed forcings: varda::cuda::DeviceRollout::run
 * (src/varda/cuda/rollout_cuda.h:40-70, rollout_cuda.cu:160-234) with RolloutRequest::replay_forcings
 * (src/varda/rollout.h:75-85); the reference's host loop Rollout::run (rollout.cpp:116-155) has the same
 * results. x0 (1, T_in, G, V_in) physical; forcings (n_steps - 1, G, F) in the config's
 * `forcings.dynamic` order (forcing s is written into the window after step s; may be NULL when
 * n_steps == 1 or F == 0); y (n_steps, G, V_out) physical receives every step's output (this rank's
 * rows on a sharded model; may be NULL); on_step (may be NULL) gets each step's rows
 * (rows, V_out) as soon as they are on the host, one step behind the GPU, valid during the call;
 * step_ms (may be NULL) [n_steps] the GPU time of each step. constants_oldest: 0 = the newest slot
 * keeps its constant inputs (ConstantSource::Newest), 1 = they come from the oldest slot
 * (ConstantSource::Oldest, rollout.h:38-41). All ranks of a sharded model call it together with the
 * same n_steps. Fails with VB_ERR_UNSUPPORTED when the config has no `forcings` section or more
 * than one output step, VB_ERR_FORMAT when the index sets do not partition the inputs. */
typedef void (*vb_step_fn)(int step, const float* y, int64_t rows, void* user);
int vb_rollout(vb_model* m, const float* x0, int n_steps, const float* forcings, float* y, int constants_oldest,
               vb_step_fn on_step, void* user, float* step_ms);

/* sizes: [T_in, G, V_in, T_out, V_out, H, C, n_proc]; input_numel = T_in G V_in, output_numel =
 * T_out G V_out (cuda/cuda_backend.h:34-35). */
int vb_sizes(const vb_model* m, int64_t out8[8]);
int vb_data_range(const vb_model* m, int64_t* lo, int64_t* hi);
/* This rank's hidden-node range [lo, hi): the processor's destination rows (all of [0, H) on one GPU). */
int vb_hidden_range(const vb_model* m, int64_t* lo, int64_t* hi);
/* Element counts of the device tensors of this rank: x/xn (T_in, G_local, V_in) and yn/y
 * (T_out, own data rows, V_out); on one GPU input_numel / output_numel (cuda_backend.h:34-35). On a
 * sharded model G_local = own data rows followed by the encoder's halo rows: the caller fills the own
 * rows of x, and vb_predict_step_device / vb_enqueue_predict fill the halo rows of every input step
 * from their owners (a collective: every rank calls them together). */
int vb_io_numel(const vb_model* m, int64_t* in, int64_t* out);

/* varda::cuda::CudaBackend device entry points (src/varda/cuda/cuda_backend.h:38-69). Pointers are
 * device pointers (fp32, contiguous); stream is a cudaStream_t (NULL = the legacy default stream). */
int vb_normalise(vb_model* m, const float* x, float* xn, void* stream);            /* :38 */
int vb_forward_normalised(vb_model* m, const float* xn, float* yn, void* stream);  /* :42 */
int vb_denormalise(vb_model* m, const float* yn, float* y, void* stream);          /* :44 */
int vb_predict_step_device(vb_model* m, const float* x, float* y, void* stream);   /* :46 */
int vb_prepare(vb_model* m);                                                       /* :50 */
int vb_use_high_priority_stream(vb_model* m);                                      /* :56 */
float* vb_device_input(vb_model* m);                                               /* :66 */
const float* vb_device_output(vb_model* m);                                        /* :67 */
void* vb_stream(vb_model* m);                                                      /* :68 */
int vb_enqueue_predict(vb_model* m);                                               /* :69 */
int vb_device(const vb_model* m);                                                  /* :71 */
size_t vb_weight_bytes(const vb_model* m);                                         /* :72 */
size_t vb_activation_bytes(const vb_model* m);                                     /* :73 */
int64_t vb_decoder_chunk_rows(const vb_model* m);                                  /* :74 */

/* Synchronises the current device and reports (then clears) the error flag a bounded device wait
 * sets when it gives up: VB_OK or VB_ERR_TIMEOUT. */
int vb_check_device(void);

/* Instrumentation, no reference counterpart (the reference profiles with external tools):
 * vb_launch_count: kernel launches issued by this library in this process so far (eager launches and
 * launches recorded into graph captures). vb_profile_forward: one eager forward pass on the model's
 * internal buffers with a CUDA event pair around every launch; writes a JSON array of
 * {"name", "ms", "flop", "bytes"} records (algorithmic FLOPs / compulsory bytes) into buf and returns
 * the length it needs (call again with a larger buffer if that exceeds len). Synchronises. */
int64_t vb_launch_count(void);
int64_t vb_profile_forward(vb_model* m, char* buf, size_t len);

/* The isolated processor block (the benchmark's C2 workload; the reference runs it only inside
 * predict_step: CpuBackend::processor, source_side then destination_side per block,
 * src/varda/cpu/backend_cpu.cpp:400-415, and the processor loop of src/varda/cuda/backend_cuda.cu:
 * 571-590 on the GPU): LN_dst then processor block `block`, `repeats` times on the same input, this
 * rank's hidden rows (vb_hidden_range). z_in: host fp32 [own hidden rows, C], or NULL to keep the
 * previous call's input (a forward pass in between overwrites it); z_out: host fp32 [own hidden rows,
 * C] receiving the block's output, or NULL. device_ms (may be NULL): device time of the runs, CUDA
 * events on the model's stream, the copies excluded. On a sharded model every run exchanges the K|V
 * halo: all ranks call it together. Synchronises. vb_profile_processor_block: one such run with an
 * event pair around every launch, records as vb_profile_forward. No reference counterpart as entry
 * points (benchmark and test instruments). */
int vb_processor_block(vb_model* m, int block, const float* z_in, float* z_out, int repeats, float* device_ms);
int64_t vb_profile_processor_block(vb_model* m, int block, char* buf, size_t len);

/* The destination partition vb_load_sharded uses for `rank` of `world` on this model file, computed
 * on the host only (no GPU): JSON with the hidden/data ranges of every rank (and the encoder's hidden
 * ranges with the row moves after the encoder; they equal the hidden ranges when VB_SHARD_ENC=0),
 * this rank's halos (global ids), its send lists per peer, and its local CSR graphs (sources in local
 * ids). Same length convention as vb_profile_forward; a negative return is minus the error class. No
 * reference counterpart (the reference runs on one GPU). */
int64_t vb_shard_plan(const char* path, int world, int rank, char* buf, size_t len);

/* ---------------------------------------------------------------- kernel-level entry points
 * The reference's internal kernel interface (src/varda/cuda/kernels.h, graph.h, gemm.h), exported
 * for unit tests and benchmarks. dtype: VB_PRECISION_FP32 (float) or VB_PRECISION_FP16 (__half
 * storage, fp32 math). All enqueue on `stream`. */

/* build_csr_by_dst (src/varda/graph.cpp:17-61), host memory: edge_index int64 [2, E], edge_attr
 * float [E, A] -> row_ptr [n_dst + 1], src [E], edge_id [E], attr_csr [E, A]. Bit-exact. */
int vb_build_csr(const int64_t* edge_index, int64_t E, const float* edge_attr, int A, int64_t n_src, int64_t n_dst,
                 int32_t* row_ptr, int32_t* src, int32_t* edge_id, float* attr_csr);

/* The rollout's state update on the device (cuda::rollout_update, src/varda/cuda/rollout_cuda.h:34-38;
 * StateUpdate::apply, rollout.cpp:70-92): window (T, rows, V_in) fp32 in place; kind [V_in] int8 =
 * 0 kept, 1 prognostic <- y[src], 2 forcing <- f[src], 3 kept from the oldest slot; y rows [0, n_own)
 * from y_own, the rest from y_halo. Device pointers. */
int vb_rollout_update(float* window, int T, int64_t rows, int V_in, const float* y_own, const float* y_halo,
                      int64_t n_own, int V_out, const float* f, int F, const int8_t* kind, const int* src,
                      void* stream);

/* One 16-byte record per CSR slot {a0, a1, a2, src} as the attention kernel reads it (the reference's
 * Engine::load_graph packing, backend_cuda.cu:323-348); host memory. round_fp16 rounds attributes. */
int vb_pack_edges(const int32_t* src, const float* attr_csr, int A, int64_t E, int round_fp16, void* out16);

/* cuda::attention<T> (src/varda/cuda/kernels.h:79-96): device pointers. edges = packed records,
 * w_e = fp32 [4, C] (edge weight columns zero padded to 3, then the edge bias). */
int vb_attention(int dtype, const int32_t* row_ptr, const void* edges, int64_t dst_lo, int64_t n_rows,
                 const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, const void* xr, int64_t ldxr,
                 void* out, int64_t ldo, const float* w_e, int C, int heads, int head_dim, void* stream);

/* vb_attention over an explicit list of destination rows (n_rows graph rows, ascending, each in
 * [0, rows of q/out)): the engine's split of a sharded processor block into interior rows (computed
 * while the halo exchange is in flight) and boundary rows. Same per-row arithmetic as vb_attention. */
int vb_attention_rows(int dtype, const int32_t* row_ptr, const void* edges, const int32_t* rows, int64_t n_rows,
                      const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, const void* xr,
                      int64_t ldxr, void* out, int64_t ldo, const float* w_e, int C, int heads, int head_dim,
                      void* stream);

/* No-allocation variant of vb_attention, no reference counterpart: same arguments and result, each
 * destination row's edges cut into `splits` parts (1..64) whose partial softmax results go to one
 * static device array of 16 MiB (its only device storage; nothing is allocated, nothing needs to start
 * at zero) and are then merged. For callers that cannot allocate device memory at call time (a process
 * whose memory pool owns the free memory, a loop that cannot take cudaMalloc's synchronisation).
 * Limit: one row's splits x (C + 5 heads) floats must fit 16 MiB (VB_ERR_UNSUPPORTED otherwise);
 * larger graphs run in several batches. Overlapping calls on one device race on the shared array:
 * order them on one stream. Make the first call on each device outside stream capture (it looks up
 * the array's device address). Destination range only; C = heads x head_dim with C a multiple of 128;
 * leading dimensions multiples of 4 elements. */
int vb_attention_split_noalloc(int dtype, const int32_t* row_ptr, const void* edges, int64_t dst_lo, int64_t n_rows,
                               const void* q, int64_t ldq, const void* k, const void* v, int64_t ldkv, const void* xr,
                               int64_t ldxr, void* out, int64_t ldo, const float* w_e, int C, int heads, int head_dim,
                               int splits, void* stream);

/* The tiled fp16 attention kernels the engine runs (no reference counterpart: the reference has only
 * the gather kernel, attention_kernel in src/varda/cuda/kernels.cu:290-419): vb_tiles_create builds the
 * destination tiles of a CSR graph (host arrays from vb_build_csr) and uploads them to the current
 * device; vb_attention_tiled runs rows [dst_lo, dst_lo + n_rows) of it (the tiles, then the rows no
 * tile covers on the gather kernel; dst_lo must start a tile, e.g. 0); same arguments and contract as
 * vb_attention, fp16 only. */
typedef struct vb_tiles vb_tiles;
int vb_tiles_create(const int32_t* row_ptr, const int32_t* src, const float* attr_csr, int A, int64_t n_src,
                    int64_t n_dst, int head_dim, vb_tiles** out);
/* The same with the tile kind: VB_TILES_SMEM (the shared-memory-staged CUDA-core kernel the engine runs
 * on the decoder graph, as vb_tiles_create) or VB_TILES_TC (the tile-sparse tensor-core kernel, which
 * the engine runs on the processor graph, or where VB_ATT_TC names a graph: tiles of up to 64 consecutive
 * rows reaching at most
 * 128 distinct sources, restarting every 64 rows; per 16-row block and head q.k and the value sums as
 * tensor-core products over the 8-column blocks that hold edges; head_dim 64 and at most 32 heads; rows
 * with a repeated source or more than 128 sources run on the gather kernel). vb_attention_tiled runs
 * whichever kind the tiles were built for. */
enum { VB_TILES_SMEM = 0, VB_TILES_TC = 1 };
/* The tile plan of a kind on the host (no device needed), for inspection and tests: counts[0] tiles,
 * counts[1] source entries, counts[2] heavy rows (left to the gather kernel); then, where the arrays
 * are non-null and sized by a first call: tiles4 [tiles][4] = {row0, nrows, src0, nsrc}, srcs (a tile's
 * slot s being srcs[src0 + s]: for VB_TILES_SMEM each tile's distinct sources in increasing order, for
 * VB_TILES_TC ordered by the first and then the last 16-row block of the tile that reads them, then by
 * first appearance along the tile's edges, padded with the last one to a
 * multiple of 4), heavy (rows), edges [E][4] (the CSR-order records {a0, a1, a2, slot or, for heavy
 * rows, source (int bits)}, attributes rounded to fp16). */
int vb_tile_plan(const int32_t* row_ptr, const int32_t* src, const float* attr_csr, int A, int64_t n_src,
                 int64_t n_dst, int kind, int64_t counts[3], int32_t* tiles4, int32_t* srcs, int32_t* heavy,
                 float* edges);
int vb_tiles_create_kind(const int32_t* row_ptr, const int32_t* src, const float* attr_csr, int A, int64_t n_src,
                         int64_t n_dst, int head_dim, int kind, vb_tiles** out);
int vb_attention_tiled(vb_tiles* t, int64_t dst_lo, int64_t n_rows, const void* q, int64_t ldq, const void* k,
                       const void* v, int64_t ldkv, const void* xr, int64_t ldxr, void* out, int64_t ldo,
                       const float* w_e, int C, int heads, int head_dim, void* stream);
void vb_tiles_free(vb_tiles* t);

/* Gemm::linear (src/varda/cuda/gemm.h): y[M, N] = A[M, K] W[N, K]^T (+ bias), then epilogue
 * 0 = none, 1 = GELU (gelu_tanh selects the tanh form), 2 = + residual R[M, N]. engine: 0 = auto
 * (tensor cores for fp16), 1 = CUDA cores, 2 = tensor cores (fp16 only; fails if not applicable).
 * The tensor-core GEMM visits its tiles in a fixed order here (the engine's own GEMMs take their next
 * tile from a counter of the model's). With VB_GEMM_SCHED=1 in the environment this entry point uses
 * the dynamic order too, on a counter kept per (device, stream, thread): then a CUDA graph holding it
 * must not run concurrently with itself or with other such launches keyed to its capture stream. Both
 * orders give the same bits. */
int vb_gemm(int dtype, int engine, const void* A, int64_t lda, const void* W, int64_t ldw, const void* bias, void* Y,
            int64_t ldy, const void* R, int64_t ldr, int64_t M, int64_t N, int64_t K, int epilogue, int gelu_tanh,
            void* stream);

/* LayerNorm fused into the GEMMs around it (fp16, tensor cores; no reference counterpart: the
 * reference runs kernels.h:49-59 as separate launches). A LayerNorm's statistics travel as segment
 * records: per row and per run of vb_ln_segment_width(N) output columns, {mean, M2} (two floats) of
 * the fp16 values stored there.
 * vb_gemm_ln: vb_gemm's tensor-core GEMM (epilogue 0, 1 or 2) that also
 *   st_out != NULL (epilogue 0 or 2): writes the output rows' records, [M, N / width] float pairs;
 *   st_in != NULL (epilogue 0 or 1): computes y = LN(A) W^T + b for W, bias folded by
 *     vb_fold_layernorm, from A's rows' records st_in ([M, nseg_in] pairs of segw_in columns,
 *     nseg_in <= 16) and the fold's column sums colsum.
 * vb_fold_layernorm: folds LN weight g and bias be (be may be NULL) into the Linear after it, in place:
 *   W[n, k] = T(W[n, k] g[k]), bias[n] = T(bias[n] + sum_k be[k] W[n, k]) (bias not NULL: zeros for
 *   a Linear without one), colsum[n] = sum_k W[n, k] after the fold (fp32).
 * vb_row_seg_stats: the records of rows of x (C columns, segments of segw) as a GEMM epilogue writes them. */
int vb_ln_segment_width(int64_t N);
int vb_gemm_ln(const void* A, int64_t lda, const void* W, int64_t ldw, const void* bias, void* Y, int64_t ldy,
               const void* R, int64_t ldr, int64_t M, int64_t N, int64_t K, int epilogue, int gelu_tanh, float* st_out,
               const float* st_in, const float* colsum, int nseg_in, int segw_in, float eps, void* stream);
int vb_fold_layernorm(void* W, int64_t ldw, int64_t N, int K, const float* g, const float* be, void* bias,
                      float* colsum, void* stream);
int vb_row_seg_stats(const void* x, int64_t ldx, int64_t rows, int C, int segw, float* st, void* stream);

/* layernorm / add_layernorm (src/varda/cuda/kernels.h:49-59); b may be NULL. */
int vb_layernorm(int dtype, const void* x, int64_t ldx, const float* w, const float* b, void* y, int64_t ldy,
                 int64_t rows, int C, float eps, void* stream);
int vb_add_layernorm(int dtype, const void* a, const void* r, void* out1, const float* w, const float* b, void* ln,
                     int64_t ld, int64_t rows, int C, float eps, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VARDA_B200_H */
