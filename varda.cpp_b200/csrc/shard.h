// Multi-GPU: the graph partitioned by destination node across the GPUs of one node, one process per
// GPU. The reference runs one GPU only; this is new (no reference counterpart).
//
// Partition. Hidden nodes are split into `world` contiguous index ranges of equal estimated cost
// (FLOPs of the node-wise GEMMs plus processor edge-gather bytes, from the config dims and
// in-degrees), and data nodes, independently, into contiguous ranges of equal estimated cost
// (encoder-source and decoder GEMMs plus decoder gathers). The forward pass is a chain of phases with
// a halo exchange between each (encoder, every processor block, decoder), so every phase is balanced
// on its own rather than each rank's total. With spatially ordered node numbering (the synthetic
// models use a Morton curve) the ranges are compact regions and the halos small; any numbering is
// correct. Optionally (encoder split) the encoder phase gets hidden ranges of its own, of equal
// estimated encoder cost (destination-side GEMMs per row, attention bytes and the source side's share
// per edge), and its output rows move to their processor owners once, right after the encoder: on a
// grid with a dense region the processor's equal-work hidden ranges put all of the region's encoder
// edges on one rank.
//
// Halos. Rank r computes the node-wise layers of its own rows only:
//   processor  K|V rows of remote hidden sources, exchanged once per block (NCCL send/recv);
//   decoder    K|V rows of remote hidden sources of its data rows, exchanged once;
//   encoder    input rows (all input steps) of remote data sources of its encoder rows, sent by
//              their owners once per forward; the encoder's source side is recomputed for them.
// Every CSR is remapped to local ids (own rows first, then the halo in global id order, which is
// also owner order) keeping each destination's stored edge order, so every destination's sums run in
// the same order as on one GPU and results are bitwise independent of the GPU count.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "config.h"
#include "engine.h"
#include "graph.h"

namespace vb {

struct HaloPlan {
    std::vector<int32_t> halo;                  // global ids of the halo sources, ascending (= owner order)
    std::vector<int64_t> recv_count;            // [world] halo rows coming from each peer
    std::vector<std::vector<int32_t>> send;     // [world] global ids of own rows each peer needs, ascending
};

struct ShardPlan {
    int world = 1, rank = 0;
    std::vector<int64_t> h_split, g_split;  // [world + 1]
    int64_t h_lo = 0, h_hi = 0, g_lo = 0, g_hi = 0;
    // The encoder's destination rows: h_split, or (encoder split) ranges of their own, balanced on the
    // encoder's work; the encoder's output rows then move to their h_split owners.
    std::vector<int64_t> e_split;  // [world + 1]
    int64_t e_lo = 0, e_hi = 0;
    // [world] global hidden-row ranges [lo, hi) (empty when hi <= lo): send_* the rows of the own
    // encoder range that peer p owns for the processor, recv_* the rows of the own hidden range that p
    // encodes; entry `rank` is the part that stays (a local copy)
    struct RowMove {
        std::vector<int64_t> send_lo, send_hi, recv_lo, recv_hi;
    } enc_move;
    HaloPlan proc, dec;
    std::vector<int32_t> enc_halo;         // global data ids read by own encoder rows but owned elsewhere
    HaloPlan enc_x;                        // the same rows as a halo plan (send lists: own data rows
                                           // other ranks read), for the rollout's per-step output exchange
    CsrGraph enc, proc_g, dec_g;           // own destination rows (enc: e_split's), sources in local ids
};

// Computes the partition and rank `rank`'s halos and local graphs from the full CSR graphs (every
// rank computes the same partition from the same file). world == 1 gives the identity plan.
// enc_split: split the encoder's destination rows on their own (e_split), else e_split = h_split.
ShardPlan make_plan(const Config& c, const CsrGraph& enc, const CsrGraph& proc, const CsrGraph& dec, int world,
                    int rank, bool enc_split = false);
// VB_SHARD_ENC=1 asks for the encoder split (default off).
bool enc_split_requested();
// JSON description of a plan (ranges, halos, send lists, local CSRs) for tests.
std::string plan_json(const ShardPlan& p, bool with_graphs);

void nccl_unique_id(void* out128);

}  // namespace vb
