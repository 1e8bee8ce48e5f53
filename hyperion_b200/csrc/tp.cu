#include "tp.h"

#include <dlfcn.h>

#include <cstring>

#include <mutex>
#include <string>
#include <vector>

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

namespace {

struct PeerTable {
    unsigned char* base[8];  // every rank's buffer, own one included (mapped into this process)
};

constexpr int kArThreads = 512;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint4 ld_cg(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// Layout of a rank's buffer: data[set][src][max] bf16, then flags[src] u32, then err u32.
__global__ void __launch_bounds__(kArThreads) oneshot_allreduce_kernel(bf16* buf, int n, PeerTable peers, int me,
                                                                       int T, size_t max_count, uint32_t epoch) {
    pdl_wait();
    const size_t set_bytes = static_cast<size_t>(T) * max_count * 2;
    const size_t slot = (epoch & 1u) * set_bytes + static_cast<size_t>(me) * max_count * 2;
    const int nv = n / 8;  // 16-byte vectors (n is a multiple of 8)
    const uint4* src = reinterpret_cast<const uint4*>(buf);
    // 1. my partial into slot `me` of every rank's current set (my own buffer included)
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
        const uint4 v = src[i];
        for (int r = 0; r < T; ++r) reinterpret_cast<uint4*>(peers.base[r] + slot)[i] = v;
    }
    __threadfence_system();
    __syncthreads();
    // 2. raise my flag on every rank (release at system scope orders the stores above)
    if (threadIdx.x < T) {
        uint32_t* flags = reinterpret_cast<uint32_t*>(peers.base[threadIdx.x] + 2 * set_bytes);
        st_release_sys(flags + me, epoch);
    }
    // 3. wait for every rank's flag of this epoch (bounded)
    __shared__ int gave_up;
    if (threadIdx.x == 0) gave_up = 0;
    __syncthreads();
    if (threadIdx.x < T) {
        const uint32_t* flags = reinterpret_cast<const uint32_t*>(peers.base[me] + 2 * set_bytes);
        bool ok = false;
        for (int it = 0; it < (1 << 24); ++it) {
            if (static_cast<int32_t>(ld_acquire_sys(flags + threadIdx.x) - epoch) >= 0) {
                ok = true;
                break;
            }
            if (it > 64) __nanosleep(64);
        }
        if (!ok) gave_up = 1;
    }
    __syncthreads();
    if (gave_up && threadIdx.x == 0) atomicAdd(reinterpret_cast<int*>(peers.base[me] + 2 * set_bytes + 4 * T), 1);
    // 4. sum the T partials in rank order (the same bits on every rank)
    const unsigned char* mine = peers.base[me] + (epoch & 1u) * set_bytes;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < T; ++r) {
            const uint4 v = ld_cg(reinterpret_cast<const uint4*>(mine + static_cast<size_t>(r) * max_count * 2) + i);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                acc[2 * k] += __uint_as_float(w[k] << 16);
                acc[2 * k + 1] += __uint_as_float(w[k] & 0xFFFF0000u);
            }
        }
        uint4 o;
        o.x = pack_bf2(f2bf(acc[0]), f2bf(acc[1]));
        o.y = pack_bf2(f2bf(acc[2]), f2bf(acc[3]));
        o.z = pack_bf2(f2bf(acc[4]), f2bf(acc[5]));
        o.w = pack_bf2(f2bf(acc[6]), f2bf(acc[7]));
        reinterpret_cast<uint4*>(buf)[i] = o;
    }
    pdl_launch_dependents();
}

}  // namespace

TpComm::~TpComm() {
    for (int r = 0; r < 8; ++r)
        if (p2p_peer_[r] && r != rank_) cudaIpcCloseMemHandle(p2p_peer_[r]);
    if (p2p_local_) cudaFree(p2p_local_);
    if (comm_) nccl().comm_destroy(comm_);
}

void TpComm::setup_p2p(size_t max_count) {
    if (!active() || size_ > 8) return;
    max_count = (max_count + 7) / 8 * 8;
    p2p_max_ = max_count;
    const size_t bytes = ll_off() + 2 * static_cast<size_t>(size_) * (max_count / 2) * 8;  // see tp.h
    HYB_CUDA(cudaMalloc(&p2p_local_, bytes));
    HYB_CUDA(cudaMemset(p2p_local_, 0, bytes));
    cudaIpcMemHandle_t mine;
    HYB_CUDA(cudaIpcGetMemHandle(&mine, p2p_local_));
    void* dev_handles = nullptr;
    HYB_CUDA(cudaMalloc(&dev_handles, sizeof(cudaIpcMemHandle_t) * (size_ + 1)));
    HYB_CUDA(cudaMemcpy(dev_handles, &mine, sizeof(mine), cudaMemcpyHostToDevice));
    all_gather_bytes(dev_handles, static_cast<char*>(dev_handles) + sizeof(mine), sizeof(mine), nullptr);
    HYB_CUDA(cudaStreamSynchronize(nullptr));
    std::vector<cudaIpcMemHandle_t> all(size_);
    HYB_CUDA(cudaMemcpy(all.data(), static_cast<char*>(dev_handles) + sizeof(mine), sizeof(mine) * size_,
                        cudaMemcpyDeviceToHost));
    cudaFree(dev_handles);
    for (int r = 0; r < size_; ++r) {
        if (r == rank_) {
            p2p_peer_[r] = p2p_local_;
        } else {
            HYB_CUDA(cudaIpcOpenMemHandle(&p2p_peer_[r], all[r], cudaIpcMemLazyEnablePeerAccess));
        }
    }
    epoch_ = 0;
    ar_seq_ = 0;
}

QmvTpFuse TpComm::next_fused_ar() {
    if (!fused_ready()) throw CudaError("fused all-reduce: peer buffers are not mapped");
    QmvTpFuse f;
    for (int r = 0; r < size_; ++r) f.peer[r] = static_cast<unsigned char*>(p2p_peer_[r]);
    f.T = size_;
    f.me = rank_;
    f.max_count = p2p_max_;
    f.ll_off = ll_off();
    f.err_off = err_off();
    // the set alternates: a rank reaches the producer of all-reduce n + 2 only after its
    // consumer of n + 1, which waited for every rank's words of n + 1, which each rank wrote
    // after its own consumer of n had finished reading set n % 2
    f.set = static_cast<int>(ar_seq_ & 1u);
    ++ar_seq_;
    f.epoch = ar_seq_;  // words start zeroed, so epoch 0 never matches
    return f;
}

void TpComm::all_reduce_small_bf16(bf16* buf, size_t count, cudaStream_t stream, bool pdl) {
    if (!active()) return;
    if (!p2p_local_ || count > p2p_max_ || count % 8 != 0 || (reinterpret_cast<uintptr_t>(buf) & 15)) {
        all_reduce_sum_bf16(buf, count, stream);
        return;
    }
    PeerTable t{};
    for (int r = 0; r < size_; ++r) t.base[r] = static_cast<unsigned char*>(p2p_peer_[r]);
    ++epoch_;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kArThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    HYB_CUDA(cudaLaunchKernelEx(&cfg, oneshot_allreduce_kernel, buf, static_cast<int>(count), t, rank_, size_, p2p_max_,
                                epoch_));
}

int TpComm::take_wait_errors(cudaStream_t stream) {
    if (!p2p_local_) return 0;
    int* err = reinterpret_cast<int*>(static_cast<unsigned char*>(p2p_local_) + err_off());
    int h = 0;
    HYB_CUDA(cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, stream));
    HYB_CUDA(cudaStreamSynchronize(stream));
    if (h) HYB_CUDA(cudaMemsetAsync(err, 0, sizeof(int), stream));
    return h;
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
