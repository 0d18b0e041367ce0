#include "comm.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.h"

namespace vb {

namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

const NcclApi& api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        a.init_rank = reinterpret_cast<decltype(a.init_rank)>(dlsym(h, "ncclCommInitRank"));
        a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
        a.send = reinterpret_cast<decltype(a.send)>(dlsym(h, "ncclSend"));
        a.recv = reinterpret_cast<decltype(a.recv)>(dlsym(h, "ncclRecv"));
        a.group_start = reinterpret_cast<decltype(a.group_start)>(dlsym(h, "ncclGroupStart"));
        a.group_end = reinterpret_cast<decltype(a.group_end)>(dlsym(h, "ncclGroupEnd"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    });
    if (!a.init_rank || !a.send || !a.recv || !a.group_start || !a.group_end || !a.get_unique_id)
        fail(kInternal, "NCCL (libnccl.so.2) could not be loaded");
    return a;
}

void check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess)
        fail(kInternal, std::string(what) + ": " + (api().error_string ? api().error_string(r) : "NCCL error"));
}

}  // namespace

void nccl_unique_id(void* out128) {
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId must be 128 bytes");
    ncclUniqueId id;
    check(api().get_unique_id(&id), "ncclGetUniqueId");
    std::memcpy(out128, &id, sizeof id);
}

Comm::Comm(int world, int rank, const void* uid) : world_(world), rank_(rank) {
    ncclUniqueId id;
    std::memcpy(&id, uid, sizeof id);
    ncclComm_t c = nullptr;
    check(api().init_rank(&c, world, id, rank), "ncclCommInitRank");
    comm_ = c;
}

Comm::~Comm() {
    if (comm_ && api().destroy) api().destroy(static_cast<ncclComm_t>(comm_));
}

void Comm::exchange(const void* send, const std::vector<int64_t>& send_off, const std::vector<int64_t>& send_count,
                    void* recv, const std::vector<int64_t>& recv_off, const std::vector<int64_t>& recv_count,
                    int elem_bytes, cudaStream_t s) {
    const ncclDataType_t t = elem_bytes == 2 ? ncclFloat16 : ncclFloat32;
    const auto* sb = static_cast<const char*>(send);
    auto* rb = static_cast<char*>(recv);
    check(api().group_start(), "ncclGroupStart");
    for (int p = 0; p < world_; ++p) {
        if (p == rank_) continue;
        if (send_count[size_t(p)])
            check(api().send(sb + send_off[size_t(p)] * elem_bytes, size_t(send_count[size_t(p)]), t, p,
                             static_cast<ncclComm_t>(comm_), s),
                  "ncclSend");
        if (recv_count[size_t(p)])
            check(api().recv(rb + recv_off[size_t(p)] * elem_bytes, size_t(recv_count[size_t(p)]), t, p,
                             static_cast<ncclComm_t>(comm_), s),
                  "ncclRecv");
    }
    check(api().group_end(), "ncclGroupEnd");
}

}  // namespace vb
