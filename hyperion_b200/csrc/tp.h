// Tensor-parallel communicator of the engine: NCCL over NVLink / NVSwitch.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2), so the library loads and all
// single-GPU paths run on machines without NCCL; only a tensor-parallel load needs it.
#pragma once

#include "common.cuh"

#include <nccl.h>

#include <cstddef>

namespace hyb {

class TpComm {
  public:
    TpComm() = default;
    ~TpComm();
    TpComm(const TpComm&) = delete;
    TpComm& operator=(const TpComm&) = delete;

    // 128 opaque bytes that rank 0 creates and every rank passes to init().
    static void unique_id(void* out);
    // Collective: every rank of the group calls it with the same id.
    void init(int rank, int size, const void* id);
    bool active() const { return size_ > 1; }
    int rank() const { return rank_; }
    int size() const { return size_; }

    // In-place bf16 sum over the ranks on `stream`.
    void all_reduce_sum_bf16(bf16* buf, size_t count, cudaStream_t stream);
    // Rank r's `bytes` land at recv + r * bytes on every rank.
    void all_gather_bytes(const void* send, void* recv, size_t bytes, cudaStream_t stream);

  private:
    ncclComm_t comm_ = nullptr;
    int rank_ = 0, size_ = 1;
};

}  // namespace hyb
