// The CUDA engine behind the hyperion_mlx.h ABI: device-resident weights, the
// per-sequence KV state and the prefill/decode forward pass.
//
// Mirrors the reference engine's structure (native/hyperion_mlx/src/model.cc,
// forward.cc, kv_cache.cc) with B200-first data layouts:
//   * q/k/v projections of a layer are fused into one packed [Nq+Nk+Nv, K/8]
//     matrix (one decode launch instead of three);
//   * gate/up are interleaved by 16-row tiles so one decode CTA produces both
//     halves of GeGLU and applies it in its epilogue;
//   * norms ride in the prologue of the next projection in decode;
//   * local KV rings are [window + 8, nkv, hd] bf16 (slot = pos % cap) and global
//     caches grow in 256-token steps, as in the reference;
//   * with tensor parallelism over TP GPUs (one process per GPU), each rank holds
//     the rows of its query/KV heads and its 1/TP of the MLP for the column-parallel
//     q/k/v and gate/up, the matching K ranges of the row-parallel o and down
//     projections (whose partial outputs are summed by an NCCL all-reduce), its KV
//     heads' caches, and 1/TP of the vocabulary for the lm_head (the greedy
//     candidates are all-gathered). Norms and the embedding table are replicated.
#pragma once

#include "common.cuh"
#include "geometry.h"
#include "kernels.h"
#include "tp.h"

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace hyb {

// Device allocation with a process-wide byte counter (telemetry).
void* dev_alloc(size_t bytes);
void dev_free(void* p);
size_t dev_active_bytes();
size_t dev_peak_bytes();
void dev_reset_peak();

template <typename T>
struct DevPtr {
    T* p = nullptr;
    size_t n = 0;
    DevPtr() = default;
    explicit DevPtr(size_t count) : p(static_cast<T*>(dev_alloc(count * sizeof(T)))), n(count) {}
    ~DevPtr() { dev_free(p); }
    DevPtr(const DevPtr&) = delete;
    DevPtr& operator=(const DevPtr&) = delete;
    DevPtr(DevPtr&& o) noexcept : p(o.p), n(o.n) { o.p = nullptr; o.n = 0; }
    DevPtr& operator=(DevPtr&& o) noexcept {
        if (this != &o) {
            dev_free(p);
            p = o.p;
            n = o.n;
            o.p = nullptr;
            o.n = 0;
        }
        return *this;
    }
    void reset(size_t count) { *this = DevPtr<T>(count); }
};

struct QLin {
    DevPtr<uint32_t> w;               // MLX layout: only while loading, freed once packed
    DevPtr<bf16> s, b;
    DevPtr<unsigned char> packed;     // the one resident copy: the packed layout
    int N = 0, K = 0;
};

// Pointers to an MLX-layout view of a matrix (codes [N, K/8] u32, scales/biases [N, K/64]).
struct MlxView {
    const uint32_t* w = nullptr;
    const bf16* s = nullptr;
    const bf16* b = nullptr;
};

struct LayerW {
    LayerKind kind = LayerKind::Sliding;
    int hd = 0, nkv = 0;
    int q_rows = 0, k_rows = 0, v_rows = 0;  // row split of the fused qkv matrix
    QLin qkv, o, gateup, down;               // gateup: interleaved 16-row tiles (gate, up)
    DevPtr<bf16> q_norm, k_norm, in_ln, post_attn, pre_ff, post_ff, scalar;
    float* inv_freq = nullptr;               // points into Model::inv_freq_*
};

struct LocalCache {
    bf16* k = nullptr;  // [cap][nkv][hd] rows inside KvState::ring_arena
    bf16* v = nullptr;
    uint32_t cap = 0, committed = 0;
    int nkv = 0, hd = 0;
    CUtensorMap tk{}, tv{};  // decode-attention tile maps of k / v (encode_kv_tensor_map)
};

struct GlobalCache {
    bf16* k = nullptr;  // [capacity][nkv][hd] rows inside KvState::global_arena
    bf16* v = nullptr;
    uint32_t capacity = 0, committed = 0;
    int nkv = 0, hd = 0;
    CUtensorMap tk{}, tv{};  // re-encoded whenever the buffers grow
};

// A state's caches live in two allocations: every ring (K then V per sliding layer) in
// ring_arena, every global cache in global_arena, which a growth replaces as a whole.
// One allocation each keeps creating, growing, cloning and freeing a state to a single
// cudaMalloc / cudaFree instead of one per layer.
struct KvState {
    DevPtr<bf16> ring_arena;
    DevPtr<bf16> global_arena;
    std::vector<LocalCache> local;
    std::vector<GlobalCache> global;
    uint32_t offset = 0;
    uint32_t last_token = 0;
    bool poisoned = false;
};

// A call that grows a global cache runs against staged buffers and publishes them only
// when it succeeds (the reference's KvGrowthTransaction, kv_cache.h:220-261,
// kv_cache.cc:68-128): the larger arena is filled from the live one and swapped in, and
// the live arena is kept here. On failure rollback restores it, the cursor and every
// commit count, so the state stays usable; on success the kept arena is freed.
// A ring (capacity window + 8) is written in place: a block of at most 8 tokens only
// overwrites slots of positions the state no longer reads, and a state at offset 0 holds
// no position a later step reads before rewriting it; a longer block on a populated state
// backs the ring arena up first.
struct KvTransaction {
    bool active = false;
    uint32_t offset = 0, last_token = 0;
    std::vector<uint32_t> local_committed, global_committed;
    struct Global {
        bf16* k = nullptr;
        bf16* v = nullptr;
        uint32_t capacity = 0;
        CUtensorMap tk{}, tv{};
    };
    DevPtr<bf16> global_arena;  // the arena the staged one replaced
    std::vector<Global> globals;
    DevPtr<bf16> ring_backup;   // a copy of ring_arena, or empty
};

// Draft tokens one verify pass may check: the speculative slack of the local rings
// (capacity window + 8). Writing positions offset..offset+8 overwrites only ring slots
// of positions at least window + 8 back, so after any acceptance every position the next
// step attends to is intact (kv.h:7-18).
constexpr int kSpecMax = 8;

struct StepOut {
    uint32_t token = 0;
    float logit = 0.f;
    bool near_tie = false;
    uint32_t topk_idx[8] = {};
    float topk_val[8] = {};
};

struct Workspace {
    int chunk_cap = 0;  // max tokens per forward
    DevPtr<bf16> h_a, h_b, h_e, xn, qkv, q, kbuf, vbuf, attn, o, gu, act, dn, logits;
    DevPtr<uint32_t> ids;
    DevPtr<float> topk_scratch;
    DevPtr<uint32_t> topk_idx;
    DevPtr<float> topk_val;
    DevPtr<uint32_t> cand;          // tensor parallel: [TP][4] gathered (idx0, val0, idx1, val1)
    DevPtr<bf16> logits_all;        // tensor parallel: the gathered full vocabulary (debug paths)
    DevPtr<unsigned char> attn_scratch;
    size_t attn_scratch_bytes = 0;
    uint32_t* h_topk_idx = nullptr;  // pinned host mirrors
    float* h_topk_val = nullptr;
    uint32_t* h_cand = nullptr;      // tensor parallel: gathered candidates
    uint32_t* h_ids = nullptr;
    int h_ids_cap = 0;
    DevPtr<unsigned char> sample;    // SampleResult of the device sampler
    SampleResult* h_sample = nullptr;  // pinned mirror
};

// Buffers of a batched decode step (sized for the largest batch seen).
struct BatchWorkspace {
    int cap = 0;                       // sequences
    DevPtr<uint32_t> x16;              // [pad(cap)][max K / 2] fp16 activation pairs
    DevPtr<bf16> logits;               // [cap][vocab_local]
    DevPtr<bf16> lm_slice;             // [cap][lm_slice_rows] one unpacked lm_head slice's GEMM output
    DevPtr<float> topk_scratch;
    DevPtr<uint32_t> topk_idx;         // [cap][8]
    DevPtr<float> topk_val;
    DevPtr<uint32_t> cand;             // tensor parallel: [cap][4] own, then [TP][cap][4] gathered
    DevPtr<unsigned char> seqs;        // [n_layers][cap] DecodeSeq of the attention launches
    DecodeSeq* h_seqs = nullptr;       // pinned staging of `seqs`
    uint32_t* h_idx = nullptr;         // pinned mirrors
    float* h_val = nullptr;
    uint32_t* h_cand = nullptr;
};

class Model {
  public:
    Model() = default;
    ~Model();

    // Load from a directory of *.safetensors (mlx-lm converted names).
    void load_dir(const Geometry& g, const std::string& dir);
    // Fill every tensor with seeded synthetic values on the device (benchmarks). With
    // tensor parallelism each rank generates exactly its shard of the TP = 1 model.
    void load_synthetic(const Geometry& g, uint64_t seed);
    // Tensor parallelism: call before loading; `id` is the 128-byte NCCL unique id
    // rank 0 created (TpComm::unique_id). The communicator is set up by the load.
    void set_tensor_parallel(int rank, int size, const void* id);
    int tp_rank() const { return tp_rank_; }
    int tp_size() const { return tp_size_; }

    std::unique_ptr<KvState> new_kv() const;
    // A copy of `src` (every cache, cursor and commit count) whose next input token is
    // `last_token`.
    std::unique_ptr<KvState> clone_kv(const KvState& src, uint32_t last_token) const;
    // Grow global caches so that `n_tokens` more tokens fit (reference
    // plan_kv_growth / GlobalKvCache::append semantics: 256-token steps).
    void reserve(KvState& kv, uint32_t n_tokens) const;
    // Device bytes a call of `n_tokens` more tokens adds while it runs (governor admission):
    // the staged global arena it grows (its full new size: the live arena stays allocated
    // until the call publishes), the ring backup of a populated state for blocks longer
    // than the ring slack, and the workspace it would newly allocate. Returns false if a
    // cache dimension would not be representable.
    bool predict_call_bytes(const KvState& kv, uint32_t n_tokens, uint64_t* bytes) const;
    // Stage the growth of a call of `n_tokens` tokens (inactive when no global cache grows).
    KvTransaction begin_kv_transaction(KvState& kv, uint32_t n_tokens) const;
    // Undo a failed call: the live buffers, cursor and commit counts come back.
    void rollback_kv_transaction(KvState& kv, KvTransaction& t) const;
    // Hard ceiling on the engine's device bytes (0 = device memory only), checked by the
    // predictive admission before any work (the governor budget of governor.h:148-186).
    void set_memory_budget(uint64_t bytes) { memory_budget_ = bytes; }
    uint64_t memory_budget() const { return memory_budget_; }

    // Prefill a prompt on a fresh state; returns the greedy sample of the last row.
    // With `sample` the last row is sampled on the device (sampler.cu) instead of taken greedily.
    StepOut prefill(KvState& kv, const uint32_t* tokens, uint32_t count, std::vector<uint16_t>* logits_out,
                    const SampleSpec* sample = nullptr);
    // One decode step at kv.offset from kv.last_token.
    StepOut decode_step(KvState& kv, std::vector<uint16_t>* logits_out, const SampleSpec* sample = nullptr);
    // One greedy decode step of `n` independent sequences together (each at its own
    // offset, from its own last_token): one weight stream per projection for the whole
    // batch. Writes outs[0..n); each state advances by one token.
    void decode_batch(KvState* const* kvs, int n, StepOut* outs);
    // Greedy speculative verify: one pass over [kv.last_token, draft[0..n)] at positions
    // kv.offset.. (1 <= n <= kSpecMax), through the batched decode stack with the rows as
    // consecutive positions of this state. outs[i] is the greedy sample after input i. The
    // longest prefix of draft that matches outs is accepted: the state commits
    // last_token and those `accepted` drafts, and its next input is outs[accepted].token,
    // so the result equals `accepted + 1` greedy decode steps. Returns `accepted`.
    int verify(KvState& kv, const uint32_t* draft, int n, StepOut* outs);

    // Attention rounding: 0 = MLX CPU-stream semantics (bf16 scores and
    // probabilities, the default), 1 = fp32 scores/probabilities (MLX's fused
    // Metal decode kernel semantics).
    void set_attention_rounding(int mode) { attn_rounding_ = mode; }
    int attention_rounding() const { return attn_rounding_; }

    // Device bytes of the weights held (packed matrices, norms, RoPE tables), the
    // algorithmic size of the quantised matrices (codes + scales + biases) and the
    // transient MLX-layout scratch the tensor-core GEMMs unpack into.
    uint64_t weight_bytes_resident() const;
    uint64_t weight_bytes_algorithmic() const;
    uint64_t unpack_scratch_bytes() const { return unpack_.n; }

    uint64_t local_kv_bytes(const KvState& kv) const;
    uint64_t global_kv_bytes(const KvState& kv) const;

    const Geometry& geometry() const { return geo_; }
    cudaStream_t stream() const { return stream_; }
    int device() const { return device_; }
    bool loaded() const { return loaded_; }

    // Exposed for tests/benchmarks through the extension ABI.
    LayerW& layer(int i) { return layers_[i]; }
    QLin& embed() { return embed_; }

  private:
    void init_common(const Geometry& g);
    // Build the packed layout of every projection and of the embedding table, then free
    // the MLX-layout copies.
    void pack_all();
    // Replace kv's global arena by one with room for `n_tokens` more tokens per global cache
    // (256-token steps), the contents copied; the old arena goes to *old. False (nothing
    // changed) when every cache already has room.
    bool grow_globals(KvState& kv, uint32_t n_tokens, DevPtr<bf16>* old) const;
    // The MLX layout of rows [row0, row0 + n) of a packed [?, K] matrix, re-derived into the
    // shared unpack scratch on `st` (valid until the next call on the same stream).
    MlxView unpack_rows(const unsigned char* packed, int K, int row0, int n, cudaStream_t st);
    void ensure_workspace(int tokens, uint32_t max_keys);
    void forward_chunk(KvState& kv, int L, uint32_t offset);  // ids already in ws_.ids
    void decode_layers(KvState& kv);
    void lm_head_rows(int B, StepOut* outs);  // B final-normed rows in ws_.xn -> greedy samples
    std::vector<int> stage_rows(KvState* const* kvs, int B, uint32_t pos_step);
    void rows_forward(int B, const std::vector<int>& keys_max, const KvState* one_seq);
    StepOut epilogue(const bf16* final_row, bool fused_prologue, const bf16* dn, const bf16* resid,
                     std::vector<uint16_t>* logits_out, const SampleSpec* sample);

    Geometry geo_;
    bool loaded_ = false;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    std::vector<LayerW> layers_;
    QLin embed_;
    DevPtr<bf16> final_norm_;
    DevPtr<float> inv_freq_local_, inv_freq_global_;
    bf16 embed_scale_{};
    int attn_rounding_ = 0;
    uint64_t memory_budget_ = 0;
    Workspace ws_;
    BatchWorkspace bws_;
    void ensure_batch_workspace(int n);
    // tensor parallelism (tp_size_ == 1: everything local)
    TpComm tp_;
    int tp_rank_ = 0, tp_size_ = 1;
    unsigned char tp_id_[128] = {};
    int heads_local_ = 0;   // query heads on this rank
    int inter_local_ = 0;   // MLP intermediate rows on this rank
    int vocab_local_ = 0;   // lm_head rows on this rank, starting at vocab0_
    int vocab0_ = 0;
    const unsigned char* lm_packed_ = nullptr;  // this rank's lm_head rows inside embed_.packed
    DevPtr<unsigned char> unpack_;              // MLX-layout scratch of the largest projection
    int lm_slice_rows_ = 0;                     // lm_head rows one unpack of the scratch holds
    QmvTpFuse last_ar_;                // the last decode layer's down_proj all-reduce (lm_head input)
};

}  // namespace hyb
