#include "tp.h"

#include <dlfcn.h>

#include <cstring>

#include <mutex>
#include <string>

namespace hyb {

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
    static NcclApi api;
    static bool loaded = false;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (!loaded) {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) throw CudaError(std::string("tensor parallelism needs NCCL: ") + dlerror());
        auto sym = [&](const char* name) {
            void* p = dlsym(h, name);
            if (!p) throw CudaError(std::string("NCCL symbol missing: ") + name);
            return p;
        };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        loaded = true;
    }
    return api;
}

void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) throw CudaError(std::string(what) + ": " + nccl().error_string(r));
}

}  // namespace

TpComm::~TpComm() {
    if (comm_) nccl().comm_destroy(comm_);
}

void TpComm::unique_id(void* out) {
    ncclUniqueId id;
    nccl_check(nccl().get_unique_id(&id), "ncclGetUniqueId");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    std::memcpy(out, &id, sizeof(id));
}

void TpComm::init(int rank, int size, const void* id) {
    if (size < 1 || rank < 0 || rank >= size) throw ArgError("tensor parallel: bad rank / size");
    rank_ = rank;
    size_ = size;
    if (size == 1) return;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    nccl_check(nccl().comm_init_rank(&comm_, size, uid, rank), "ncclCommInitRank");
}

void TpComm::all_reduce_sum_bf16(bf16* buf, size_t count, cudaStream_t stream) {
    if (!active()) return;
    nccl_check(nccl().all_reduce(buf, buf, count, ncclBfloat16, ncclSum, comm_, stream), "ncclAllReduce");
}

void TpComm::all_gather_bytes(const void* send, void* recv, size_t bytes, cudaStream_t stream) {
    if (!active()) {
        if (send != recv) HYB_CUDA(cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, stream));
        return;
    }
    nccl_check(nccl().all_gather(send, recv, bytes, ncclUint8, comm_, stream), "ncclAllGather");
}

}  // namespace hyb
