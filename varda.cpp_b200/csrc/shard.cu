// Multi-GPU loader (destination partition + halo exchange). Filled in by the sharded engine.
#include "common.h"
#include "shard.h"

namespace vb {

std::unique_ptr<Model> load_sharded_model(const std::string&, const Options&) {
    fail(kUnsupported, "sharded models are not available in this build");
}

void nccl_unique_id(void*) { fail(kUnsupported, "NCCL is not available in this build"); }

}  // namespace vb
