// Host-side launch interface of every sm_100a kernel in this library.
//
// All pointers are device pointers; all tensors are dense row-major. bf16
// values travel as __nv_bfloat16. Every launcher enqueues on `stream` and
// throws hyb::CudaError on a launch failure.
#pragma once

#include "common.cuh"

namespace hyb {

// ---------------------------------------------------------------- quantized matmul
// Affine Q4/g64: y[m, n] = sum_k x[m, k] * (s[n, k/64] * q[n, k] + b[n, k/64]),
// q[n, 8j+i] = bits [4i, 4i+4) of w[n, j]. x bf16 [M, K], w u32 [N, K/8],
// s/b bf16 [N, K/64], y bf16 [M, N]. K must be a multiple of 64.

// Prologue applied to the activation before the batch-1 qmv.
enum class QmvPrologue : int {
    kNone = 0,       // x is used as given
    kNorm = 1,       // x <- rms_norm(x, norm_w)
    kResidNorm = 2,  // h = resid + rms_norm(x, post_w) [* scalar]; written to h_out by CTA 0;
                     // x <- rms_norm(h, norm_w)
};
// Epilogue of the batch-1 qmv.
enum class QmvEpilogue : int {
    kStore = 0,   // y[n] = bf16(acc)
    kGeglu = 1,   // rows are (gate, up) interleaved by 16-row tiles: y[n] = bf16(gelu(g) * u)
};

// Tensor-parallel all-reduce fused into the decode qmvs over NVLink peer memory, in words
// that carry their own flag: a row-parallel qmv (ar_mode 1) writes its bf16 output rows in
// pairs as 8-byte words {row 2k, row 2k + 1, epoch} into slot (set, me) of every rank's
// receive buffer (IPC-mapped into every process, own included); an aligned 8-byte store is
// single-copy atomic, so a word whose epoch matches carries its data, and no fence or
// counter is needed. The next qmv (ar_mode 2) spins (bounded) on each word of every source
// until its epoch is this all-reduce's, then uses x = bf16(sum over sources in rank order)
// as its input: the same bits on every rank. Receive buffer: [2 sets][T sources]
// [max_count / 2] u64 words at ll_off, a wait-error counter at err_off.
struct QmvTpFuse {
    unsigned char* peer[8] = {};
    int T = 0, me = 0;
    int set = 0;                // receive set of this all-reduce
    unsigned epoch = 0;         // sequence number of this all-reduce (>= 1) carried by its words
    size_t max_count = 0;       // elements per (set, source) slot (even)
    size_t ll_off = 0;          // byte offset of the words in a buffer
    size_t err_off = 0;         // byte offset of the wait-error counter
};

struct QmvParams {
    const bf16* x = nullptr;          // [K] activation (or the branch output for kResidNorm)
    const uint32_t* w = nullptr;      // [N, K/8]
    const bf16* s = nullptr;          // [N, K/64]
    const bf16* b = nullptr;          // [N, K/64]
    bf16* y = nullptr;                // [N] (or [N/2] for kGeglu)
    int K = 0;
    int N = 0;
    QmvPrologue prologue = QmvPrologue::kNone;
    QmvEpilogue epilogue = QmvEpilogue::kStore;
    // prologue operands
    const bf16* norm_w = nullptr;     // [K] weight of the final norm in the prologue
    const bf16* resid = nullptr;      // [K] residual stream (kResidNorm)
    const bf16* post_w = nullptr;     // [K] norm applied to x before the residual add
    const bf16* scalar = nullptr;     // [1] layer_scalar multiplied after the add, or null
    bf16* h_out = nullptr;            // [K] new residual, written by CTA 0
    float eps = 1e-6f;
    const void* packed = nullptr;     // packed resident layout (launch_qmv_packed); w/s/b unused then
    // fused tensor-parallel all-reduce: 0 none, 1 produce (store rows to every rank),
    // 2 consume (x = the all-reduced rows); packed path, K and N <= ar.max_count
    int ar_mode = 0;
    QmvTpFuse ar;
};

void launch_qmv(const QmvParams& p, cudaStream_t stream, bool pdl = false);

// Packed resident layout for the TMA-streamed qmv (see qmv_packed.cu): bytes for
// an [N, K] matrix, the repack from the MLX layout, and the kernel itself.
size_t qmv_packed_bytes(int K, int N);
void launch_qmv_pack(const uint32_t* w, const bf16* s, const bf16* b, int K, int N, void* packed,
                     cudaStream_t stream);
void launch_qmv_packed(const QmvParams& p, cudaStream_t stream, bool pdl = false);
// The MLX layout of a packed matrix's N rows (the inverse of launch_qmv_pack).
void launch_qmv_unpack(const void* packed, int K, int N, uint32_t* w, bf16* s, bf16* b, cudaStream_t stream);
// Embedding gather (+ dequantise, x scale) of L token rows from a packed [N, H] table.
void launch_embed_packed(const uint32_t* ids, int L, const void* packed, int H, int N, bf16 scale, bf16* out,
                         cudaStream_t stream);

// Batched decode qmv (qmv_batched.cu): B <= kMaxDecodeBatch sequences over the packed
// layout, one weight stream for the whole batch. x16 is the activation batch converted by
// launch_qmv_batched_x16 (qmv_batch_x16_words(B, K) u32, tiled per 512-code unit); y is
// [B][ldy] (N/2 columns with the GeGLU epilogue over the interleaved gate/up matrix).
constexpr int kMaxDecodeBatch = 64;
struct QmvBatchParams {
    const uint32_t* x16 = nullptr;
    const void* packed = nullptr;
    bf16* y = nullptr;
    int K = 0, N = 0, B = 0, ldy = 0;
    bool geglu = false;
};
int qmv_batch_pad(int B);
size_t qmv_batch_x16_words(int B, int K);
void launch_qmv_batched_x16(const bf16* x, int B, int ldx, int K, uint32_t* x16, cudaStream_t stream);
void launch_qmv_batched(const QmvBatchParams& p, cudaStream_t stream, bool pdl = false);
int64_t read_qmvb_wait_timeouts();

// Prefill GEMM for M >= 2 (tensor cores; fp16 operands, fp32 accumulation).
// Prefill qmm on tcgen05 tensor cores with TMEM accumulators (qmm_tc.cu): 128x256 output
// tiles, f16 operands dequantised in shared memory, fp32 accumulation.
bool qmm_tc_supported(int M, int K, int N);
void launch_qmm_tc(const bf16* x, const uint32_t* w, const bf16* s, const bf16* b, bf16* y, int M, int K, int N,
                   cudaStream_t stream, bool geglu = false);
// geglu: W is the interleaved gate/up matrix (16-row tiles) and y [M, N/2] receives
// GeGLU(gate, up) from the epilogue; shapes the split-K plan would take are not supported.
bool qmm_tc_geglu_supported(int M, int K, int N);
int64_t read_qmm_wait_timeouts();
// Legacy prefill qmm on mma.sync (qmm.cu).
void launch_qmm(const bf16* x, const uint32_t* w, const bf16* s, const bf16* b, bf16* y,
                int M, int K, int N, cudaStream_t stream);

// Dispatcher used by the op-level ABI: qmv for M == 1, qmm otherwise.
void launch_quantized_matmul(const bf16* x, const uint32_t* w, const bf16* s, const bf16* b,
                             bf16* y, int M, int K, int N, cudaStream_t stream);

// ---------------------------------------------------------------- elementwise / norms
// out[l, :] = bf16(bf16(s*q + b) * embed_scale) for ids[l] rows of the packed table.
void launch_embed(const uint32_t* ids, int L, const uint32_t* w, const bf16* s, const bf16* b,
                  int H, bf16 embed_scale, bf16* out, cudaStream_t stream);

// Row-wise RMSNorm: out = bf16(bf16(x * inv) * w) (w may be null), rows of length D.
void launch_rms_norm(const bf16* x, const bf16* w, bf16* out, int rows, int D, float eps,
                     cudaStream_t stream);

// h = bf16(resid + norm(x, post_w)); h = bf16(h * scalar) if scalar; out_h = h;
// out_n = norm(h, next_w) if next_w.
void launch_resid_norm(const bf16* x, const bf16* post_w, const bf16* resid,
                       const bf16* scalar, bf16* out_h, const bf16* next_w, bf16* out_n,
                       int rows, int D, float eps, cudaStream_t stream);

// act[l, n] = bf16(gelu_tanh(gate[l, n]) * up[l, n]) with the reference's bf16 op rounding.
void launch_geglu(const bf16* gate, const bf16* up, bf16* act, int rows, int N, int ld_in,
                  cudaStream_t stream);

// Per token l and head: QK-norm (q/k with weights, v without), RoPE on q and k at
// position pos0 + l, and the cache writes. qkv is [L, ld] with q at column 0,
// k at q_cols, v at q_cols + kv_cols (v_from_k: v reads the k columns).
struct QkvPostParams {
    const bf16* qkv = nullptr;
    int L = 0, ld = 0;
    int n_heads = 0, n_kv = 0, hd = 0;
    bool v_from_k = false;
    const bf16* q_norm = nullptr;
    const bf16* k_norm = nullptr;
    const float* inv_freq = nullptr;   // [hd/2], 0 = identity pair
    int pos0 = 0;
    float eps = 1e-6f;
    bf16* q_out = nullptr;             // [L, n_heads, hd]
    bf16* k_out = nullptr;             // optional contiguous [L, n_kv, hd]
    bf16* v_out = nullptr;
    bf16* k_cache = nullptr;           // optional [cap, n_kv, hd]; slot = (pos0 + l) % cap
    bf16* v_cache = nullptr;
    int cache_cap = 0;
    int cache_first = 0;               // only tokens l >= cache_first are written to the cache
};
void launch_qkv_post(const QkvPostParams& p, cudaStream_t stream);

// Gather cache rows for positions [pos0, pos0 + n) (slot = pos % cap) into dst [n, n_kv, hd].
void launch_gather_ring(const bf16* cache, int cap, int pos0, int n, int row_elems, bf16* dst,
                        cudaStream_t stream);

// logits -> bf16 softcap (cap > 0) in place, then per-block top candidates for argmax/top-k.
// Final result: idx/val of the TOPK largest (first index wins ties), plus top2 for near-tie.
// Seeded stochastic sampling of one post-softcap logit row on the device (sampler.cu):
// temperature, top-p, min-p and top-k filters, softmax and a std::mt19937_64-seeded
// inverse-CDF draw with the reference's step order (forward.cc:191-322). Filters are off at
// 0 (top_p also at >= 1); temperature must be > 0. One CTA; no scratch memory.
struct SampleSpec {
    float temperature = 1.f, top_p = 0.f, min_p = 0.f;
    int top_k = 0;
    uint64_t seed = 0;
};
struct SampleResult {
    uint32_t token;
    float logit;                      // the sampled token's raw (post-softcap) logit
    uint32_t topk_idx[8];             // the 8 largest raw logits, value desc, index asc
    float topk_val[8];
    uint32_t topk_count;
    uint32_t kept;                    // tokens the filters kept
    float u, sz;                      // the draw and the kept tokens' total weight
};
void launch_sample(const bf16* logits, int n, const SampleSpec& spec, SampleResult* out, cudaStream_t stream);

void launch_softcap_topk(bf16* logits, int N, float cap, float* scratch, int scratch_floats,
                         uint32_t* out_idx, float* out_val, cudaStream_t stream);
int softcap_topk_scratch_floats(int N);
// The same over `rows` rows of a [rows][ld] logits batch: the winner and runner-up of row r
// at out_* + kTopkRowStride * r; scratch of rows * softcap_topk_scratch_floats(N) floats.
constexpr int kTopkRowStride = 8;
void launch_softcap_topk_rows(bf16* logits, int rows, long long ld, int N, float cap, float* scratch,
                              size_t scratch_floats, uint32_t* out_idx, float* out_val, cudaStream_t stream);

// ---------------------------------------------------------------- attention
// Decode (one query token): q [H, hd]; caches [cap, Hkv, hd]; keys are the last
// n_keys committed positions ending at `last_pos` (slot = pos % cap).
struct DecodeAttnParams {
    const bf16* q = nullptr;
    const bf16* k_cache = nullptr;
    const bf16* v_cache = nullptr;
    bf16* out = nullptr;       // [H, hd]
    int n_heads = 0, n_kv = 0, hd = 0;
    int cap = 0;
    int last_pos = 0;          // absolute position of the query (the newest key)
    int n_keys = 0;            // keys at positions last_pos - n_keys + 1 .. last_pos
    float scale = 1.0f;
    float softcap = 0.0f;
    int rounding = 0;          // 0: MLX CPU-stream (bf16 scores and probabilities), 1: none
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
};
size_t decode_attn_scratch_bytes(int n_heads, int n_kv, int hd, int max_keys);
void launch_decode_attn(const DecodeAttnParams& p, cudaStream_t stream);
// The same attention with its scratch in a fixed file-scope device buffer
// (p.scratch / p.scratch_bytes are ignored); throws ArgError above the limit.
void launch_decode_attn_noalloc(DecodeAttnParams p, cudaStream_t stream);
size_t decode_attn_noalloc_limit_bytes();

// Fused single-token decode attention (attention_fused.cu): from the raw projection
// row qkv (q | k | v, or q | k with v_from_k) it normalises and rotates q and the new
// k, normalises the new v, appends k/v at slot pos % cap, and attends over the
// n_keys positions pos - n_keys + 1 .. pos. One thread-block cluster per KV head.
// One sequence of a batched fused decode attention launch (device memory, 64-byte
// aligned array; the tensor maps are read by TMA from there).
struct alignas(64) DecodeSeq {
    CUtensorMap tk, tv;       // encode_kv_tensor_map of k_cache / v_cache
    const bf16* qkv = nullptr;  // this sequence's projection row
    bf16* out = nullptr;        // [n_heads, hd]
    bf16* k_cache = nullptr;
    bf16* v_cache = nullptr;
    int cap = 0, pos = 0, n_keys = 0, pad = 0;
};

struct DecodeFusedParams {
    const bf16* qkv = nullptr;
    bool v_from_k = false;
    const bf16* q_norm = nullptr;
    const bf16* k_norm = nullptr;
    const float* inv_freq = nullptr;
    float eps = 1e-6f;
    bf16* k_cache = nullptr;  // [cap, n_kv, hd]
    bf16* v_cache = nullptr;
    int cap = 0;
    int pos = 0;
    int n_keys = 0;
    int n_heads = 0, n_kv = 0, hd = 0;
    float scale = 1.0f;
    float softcap = 0.0f;
    int rounding = 0;
    bf16* out = nullptr;      // [n_heads, hd]
    // Optional pre-encoded tensor maps of k_cache / v_cache (encode_kv_tensor_map);
    // encoded per launch when null.
    const CUtensorMap* tmap_k = nullptr;
    const CUtensorMap* tmap_v = nullptr;
    // Batched launch (launch_decode_attn_fused_batch): per-sequence fields of n_seq
    // sequences on the device; qkv/out/caches/cap/pos/n_keys/tensor maps above unused.
    const DecodeSeq* seqs = nullptr;
    int n_seq = 0;
    // The newest position's K/V are already in the caches (appended by an earlier launch,
    // e.g. rows of one sequence at consecutive positions): the kernel neither computes nor
    // appends them and reads every key from the caches. Such a launch must not use PDL.
    bool kv_ready = false;
};
// Tiled TMA tensor map (rank <= 5): dims innermost first, strides in bytes for dims
// 1..rank-1, box in elements; no interleave, zero fill out of bounds (tma_host.cu).
void encode_tma(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// 3-D tensor map over a [cap, n_kv, hd] bf16 cache whose box is 64 consecutive
// slots x 64 dims of one KV head, 128-byte swizzled (the fused decode attention's
// tile is hd/64 such boxes).
void encode_kv_tensor_map(CUtensorMap* map, const bf16* cache, int cap, int n_kv, int hd);
void launch_decode_attn_fused(const DecodeFusedParams& p, cudaStream_t stream, bool pdl = false);
// Whether the fused kernel's shared-memory plan holds n_keys scores (else use the
// split-K path above).
// Batched fused decode attention: one launch over `seqs` (device array of n_seq, built by
// the caller) sharing layer weights and shapes; n_keys_max sizes the shared-memory plan.
void launch_decode_attn_fused_batch(const DecodeFusedParams& p, int n_keys_max, cudaStream_t stream, bool pdl);
bool decode_attn_fused_fits(int n_heads, int n_kv, int hd, int n_keys);

// Bounded mbarrier waits that gave up on the current device (never expected):
// qmv_packed.cu and attention_fused.cu each keep a counter.
int64_t read_qmv_wait_timeouts();
int64_t read_attn_wait_timeouts();

// Prefill: q [Lq, H, hd] at positions q_pos0 + i; k/v [Lk, Hkv, hd] at k_pos0 + j.
struct PrefillAttnParams {
    const bf16* q = nullptr;
    const bf16* k = nullptr;
    const bf16* v = nullptr;
    bf16* out = nullptr;
    int Lq = 0, Lk = 0, n_heads = 0, n_kv = 0, hd = 0;
    int q_pos0 = 0, k_pos0 = 0;
    int window = 0;            // 0 = full causal
    float scale = 1.0f;
    float softcap = 0.0f;
    int rounding = 0;
};
void launch_prefill_attn(const PrefillAttnParams& p, cudaStream_t stream);
// The tcgen05 version (attention_tc.cu), which launch_prefill_attn uses when it applies
// (head_dim 64/128/256, 16-byte aligned operands); the mma.sync kernel otherwise.
bool prefill_attn_tc_supported(const PrefillAttnParams& p);
void launch_prefill_attn_tc(const PrefillAttnParams& p, cudaStream_t stream);
void launch_prefill_attn_mma(const PrefillAttnParams& p, cudaStream_t stream);
int64_t read_attn_tc_wait_timeouts();

}  // namespace hyb
