// Tensor-parallel communicator of the engine: NCCL over NVLink / NVSwitch.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2), so the library loads and all
// single-GPU paths run on machines without NCCL; only a tensor-parallel load needs it.
#pragma once

#include "common.cuh"
#include "kernels.h"

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

    // In-place bf16 sum over the ranks on `stream` (NCCL).
    void all_reduce_sum_bf16(bf16* buf, size_t count, cudaStream_t stream);

    // One-shot all-reduce for small decode messages over NVLink peer memory: each rank
    // stores its partial into every peer's receive buffer (IPC-mapped, plain stores),
    // raises a release flag, waits (bounded) for all flags and sums in rank order, so
    // every rank gets the same bits. setup_p2p is collective; messages above the set-up
    // size (or without peer access) go through NCCL.
    void setup_p2p(size_t max_count);
    void all_reduce_small_bf16(bf16* buf, size_t count, cudaStream_t stream, bool pdl);
    // Number of flag waits that gave up since the last call (then resets it); a wait that
    // gives up leaves that step's result undefined but never hangs the GPU.
    int take_wait_errors(cudaStream_t stream);
    // Fused all-reduce in the decode qmvs (QmvTpFuse): available once setup_p2p mapped the
    // peers' buffers. next_fused_ar() describes the next all-reduce of up to the set-up
    // count (every rank calls it in the same order, so the receive set and the epoch agree).
    bool fused_ready() const { return p2p_local_ != nullptr; }
    QmvTpFuse next_fused_ar();
    // Rank r's `bytes` land at recv + r * bytes on every rank.
    void all_gather_bytes(const void* send, void* recv, size_t bytes, cudaStream_t stream);

  private:
    ncclComm_t comm_ = nullptr;
    int rank_ = 0, size_ = 1;
    // local buffer: one-shot all-reduce data [2 sets][size][max] bf16, its flags [size] u32,
    // the wait-error counter u32, then (16-byte aligned, at ll_off) the fused all-reduce's
    // flagged words [2 sets][size][max / 2] u64
    void* p2p_local_ = nullptr;
    void* p2p_peer_[8] = {};
    size_t p2p_max_ = 0;
    uint32_t epoch_ = 0;
    uint32_t ar_seq_ = 0;  // fused all-reduces issued
    size_t err_off() const { return 2 * static_cast<size_t>(size_) * p2p_max_ * 2 + 4 * static_cast<size_t>(size_); }
    size_t ll_off() const { return (err_off() + 4 + 15) / 16 * 16; }
};

}  // namespace hyb
