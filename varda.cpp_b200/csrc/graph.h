// Static graphs in destination-major CSR layout, built once at load time, and their packed device
// form. The CSR build is the reference's build_csr_by_dst (src/varda/graph.cpp:17-61, graph.h:15-25)
// restated: a stable counting sort of the stored edges by destination, so per-destination sums
// visit edges in stored order. Bit-exact by construction (pure integer work).
#pragma once

#include <cstdint>
#include <vector>

#include "safetensors.h"

namespace vb {

struct CsrGraph {
    int64_t n_src = 0, n_dst = 0, n_edges = 0;
    int attr_dim = 0;
    std::vector<int32_t> row_ptr;  // [n_dst + 1]
    std::vector<int32_t> src;      // [n_edges]
    std::vector<int32_t> edge_id;  // [n_edges] stored index of each CSR slot
    std::vector<float> attr;       // [n_edges, attr_dim]
    int32_t max_degree() const;
};

// edge_index: I64 or I32 [2, E] (row 0 source, row 1 destination); edge_attr: F32 [E, A].
CsrGraph build_csr_by_dst(const TensorView& edge_index, const TensorView& edge_attr, int64_t n_src, int64_t n_dst);
// Same on raw host arrays (edge_index int64 [2, E]); used by the C ABI.
CsrGraph build_csr_by_dst(const int64_t* edge_index, int64_t E, const float* edge_attr, int A, int64_t n_src,
                          int64_t n_dst);

// One 16-byte record per CSR slot: {a0, a1, a2, bitcast<float>(src)}, attributes zero-padded to
// three and, in fp16 mode, rounded to fp16 as autocast does to the edge Linear's input.
struct EdgeRec {
    float a0, a1, a2;
    int32_t src;
};
static_assert(sizeof(EdgeRec) == 16, "edge record must be 16 bytes");
std::vector<EdgeRec> pack_edges(const CsrGraph& g, bool round_fp16);

// Destination tiles for the shared-memory-staged attention: consecutive destination rows grouped
// while the union of their sources stays within `max_src` and the tile within `max_rows` rows. A row
// whose own distinct sources exceed `max_src`, or whose degree exceeds `max_deg`, is "heavy" and left to
// the gather kernel; tiles never straddle a multiple of `chunk_rows` (the decoder's destination
// chunks; 0: no chunking). Per tile the
// distinct sources are listed (ascending), and every edge of a tiled row carries, in place of its
// source id, the slot of that source in its tile's list.
struct TilePlan {
    std::vector<int32_t> row0, nrows, src0, nsrc;  // per tile
    std::vector<int32_t> srcs;                     // distinct sources of every tile, concatenated
    std::vector<EdgeRec> edges;                    // CSR order; src = slot for tiled rows
    std::vector<int32_t> heavy;                    // rows left to the gather kernel
    int max_nsrc = 0;
};
// Tiles of consecutive destination rows with at most max_src distinct sources, max_rows rows and
// max_edges edges; a row with more than max_src distinct sources, more than max_edges edges or more
// than max_row_edges edges (0: no limit) is heavy (left to the gather kernel). Tiles never span a
// multiple of chunk_rows (0: no chunking). Slots number a tile's sources in increasing source order;
// with sort_by_slot each tiled row's records are stably sorted by slot.
TilePlan make_tiles(const CsrGraph& g, int max_src, int max_rows, int max_edges, int64_t chunk_rows, bool round_fp16,
                    int max_row_edges = 0, bool sort_by_slot = false);

// Tiles of the tensor-core edge attention (attention_tc.cu): runs of at most kTcRows consecutive
// destination rows whose edges reach at most kTcMaxSrc distinct sources and number at most
// kTcMaxEdges, grown greedily; a tile that a limit cuts after more than 16 rows ends at its last whole
// 16-row block (the kernel's unit of work). A tile's sources are numbered (its "slots") by the first 16-row block of the tile that
// reads them, then by the last one, then by first appearance along the tile's CSR edges, so the
// numbering depends only on the tile's rows, not on how the graph's nodes are numbered; tiles restart at every multiple of align_rows (so a graph split into row ranges at such
// multiples gets the same tiles). Rows with more than kTcMaxSrc distinct sources or kTcMaxEdges edges,
// or with a source that appears twice, are "heavy": no tile covers them (the gather kernel does).
constexpr int kTcRows = 64, kTcMaxSrc = 128, kTcMaxEdges = 1024;
// Row alignment of the tile restarts (the multi-GPU destination split rounds its hidden ranges to it).
constexpr int64_t kTcAlignRows = 64;
// Per-tile record block (16-byte aligned), in this order:
//   per 16-row block b (at kTcBlockOff + 32 b): u8 chunk count n_b, u8 chunk base (index of the block's
//       first chunk in the tile), then 2 n_b u8 column-block indices: the block's 8-slot column blocks
//       that hold edges, in pairs (one pair per chunk; an odd count padded with a repeat that holds no
//       edge);
//   per chunk c (at kTcMaskOff + 32 c): per lane l of a warp one u8 mask: bit e set when fragment
//       position e of lane l in the chunk is an edge. Lane l = 4 r + t holds positions
//       e = 4 k + 2 h + i: column block k of the chunk (first, second), row r + 8 h of the block, slot
//       column 2 t + i of the column block;
//   at attr_off = kTcMaskOff + 32 n_chunks, per chunk 1536 bytes: per lane 48 bytes, for each pair
//       p = e / 2 of positions (same row, adjacent columns) three fp16x2 words (a0, a1, a2) x
//       (position 2p, position 2p + 1), zero where there is no edge.
// The head and masks ([0, attr_off)) are what the kernel stages in shared memory; the attributes it
// reads from global memory, one coalesced 48-byte run per lane and chunk.
constexpr int kTcBlockOff = 0, kTcMaskOff = 128, kTcChunkAttr = 1536, kTcMaxChunks = 4 * (kTcMaxSrc / 16);
struct TcTile {
    int32_t row0, nrows, nsrc, src_off;               // rows [row0, row0 + nrows); sources srcs[src_off, + nsrc)
    int32_t blob_off, blob_bytes, n_edges, attr_off;  // record block: byte offset, size; attributes offset
};
static_assert(sizeof(TcTile) == 32, "tile descriptor must be 32 bytes");
struct TcPlan {
    std::vector<TcTile> tiles;
    std::vector<int32_t> srcs;  // per tile, padded with its last source to a multiple of 4
    std::vector<uint8_t> blob;  // record blocks
    std::vector<int32_t> heavy;
};
// Attributes are rounded to fp16 (the plan serves the fp16 path only).
TcPlan make_tc_tiles(const CsrGraph& g, int64_t align_rows);

}  // namespace vb
