// Multi-GPU: the graph partitioned by destination node across the GPUs of one node, one process
// per GPU, halo K/V exchange between processor blocks.
#pragma once

#include <memory>
#include <string>

#include "engine.h"

namespace vb {

std::unique_ptr<Model> load_sharded_model(const std::string& path, const Options& opts);
void nccl_unique_id(void* out128);

}  // namespace vb
