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
// correct.
//
// Halos. Rank r computes the node-wise layers of its own rows only:
//   processor  K|V rows of remote hidden sources, exchanged once per block (NCCL send/recv);
//   decoder    K|V rows of remote hidden sources of its data rows, exchanged once;
//   encoder    input rows of remote data sources of its hidden rows, uploaded from the host with
//              the rank's own input rows (no device exchange: the encoder's source side is
//              recomputed for them).
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
    HaloPlan proc, dec;
    std::vector<int32_t> enc_halo;         // global data ids read by own hidden rows but owned elsewhere
    HaloPlan enc_x;                        // the same rows as a halo plan (send lists: own data rows
                                           // other ranks read), for the rollout's per-step output exchange
    CsrGraph enc, proc_g, dec_g;           // own destination rows, sources in local ids
};

// Computes the partition and rank `rank`'s halos and local graphs from the full CSR graphs (every
// rank computes the same partition from the same file). world == 1 gives the identity plan.
ShardPlan make_plan(const Config& c, const CsrGraph& enc, const CsrGraph& proc, const CsrGraph& dec, int world,
                    int rank);
// JSON description of a plan (ranges, halos, send lists, local CSRs) for tests.
std::string plan_json(const ShardPlan& p, bool with_graphs);

void nccl_unique_id(void* out128);

}  // namespace vb
