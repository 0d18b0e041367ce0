// NCCL communicator for the multi-GPU partition, loaded at run time (dlopen "libnccl.so.2": the
// library already in the process, e.g. torch's, or the system one), so single-GPU use needs none.
// Only point-to-point send/recv is used: the halo exchanges of the destination partition.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

namespace vb {

class Comm {
public:
    Comm(int world, int rank, const void* unique_id128);
    ~Comm();
    Comm(const Comm&) = delete;
    Comm& operator=(const Comm&) = delete;
    int world() const { return world_; }
    int rank() const { return rank_; }
    // Grouped point-to-point exchange on s: for every peer p, send send_count[p] elements starting at
    // send + send_off[p] and receive recv_count[p] elements into recv + recv_off[p] (element counts
    // and offsets in elements of `elem_bytes` = 2 (fp16) or 4 (fp32)).
    void exchange(const void* send, const std::vector<int64_t>& send_off, const std::vector<int64_t>& send_count,
                  void* recv, const std::vector<int64_t>& recv_off, const std::vector<int64_t>& recv_count,
                  int elem_bytes, cudaStream_t s);

private:
    int world_, rank_;
    void* comm_ = nullptr;
};

void nccl_unique_id(void* out128);

}  // namespace vb
