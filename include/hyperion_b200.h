/*
 * hyperion_b200.h - extension entry points of the B200 engine library.
 *
 * These sit beside the 14-function hyperion_mlx.h ABI (which they do not change)
 * and expose the engine's kernels one by one, in plain C with device pointers,
 * so that tests and benchmarks can drive each hot-path op directly. Each entry
 * point names the reference interface it replaces. All pointers are CUDA device
 * pointers unless a comment says "host"; `stream` is a cudaStream_t (NULL =
 * the legacy default stream). bf16 tensors are passed as `void*`.
 *
 * Every function returns a HypStatus and records a message for hyp_last_error
 * on failure: INVALID_ARGUMENT for bad shapes or null pointers, UNSUPPORTED for
 * shapes the kernels do not implement, INTERNAL for CUDA errors.
 */
#ifndef HYPERION_B200_H
#define HYPERION_B200_H

#include <stddef.h>
#include <stdint.h>

#include "hyperion_mlx.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Library build identity: writes a NUL-terminated string like "hyperion_b200 sm_100a". */
HypStatus hyb_build_info(char* buffer, size_t buffer_len);

/*
 * Affine Q4/g64 quantized matmul, y = x * dequant(w)^T.
 * Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true,
 * group_size=64, bits=4, "affine") as called by QuantizedLinear::apply
 * (native/hyperion_mlx/src/weights.h:26-37).
 *   x: bf16 [M, K]; w: u32 [N, K/8] (code i of word j of row n = q[n, 8j+i],
 *   bits [4i, 4i+4)); scales, biases: bf16 [N, K/64]; y: bf16 [M, N].
 *   M == 1 runs the decode qmv kernel, M > 1 the prefill GEMM.
 * group_size must be 64 and bits 4 (UNSUPPORTED otherwise); K a multiple of 64.
 */
HypStatus hyb_quantized_matmul(const void* x, const uint32_t* w, const void* scales,
                               const void* biases, void* y, int64_t M, int64_t K, int64_t N,
                               int32_t group_size, int32_t bits, void* stream);

/*
 * Single-token attention over a KV cache, the q_len == 1 case of
 * mx::fast::scaled_dot_product_attention(q, k, v, scale, bool mask)
 * (native/hyperion_mlx/src/forward.cc:498-504) together with the cache read that
 * feeds it (forward.cc:474-494, kv_cache.cc:251-265).
 *   q: bf16 [n_heads, head_dim]; k_cache, v_cache: bf16 [capacity, n_kv, head_dim]
 *   where absolute position p lives in slot p % capacity (a ring for sliding
 *   layers; capacity >= positions for a global cache). The query sits at
 *   last_pos and attends to the n_keys positions last_pos - n_keys + 1 .. last_pos.
 *   out: bf16 [n_heads, head_dim]. softcap > 0 applies softcap * tanh(s / softcap)
 *   to the scores (off for Gemma 4). rounding 0 reproduces MLX's CPU-stream
 *   rounding (bf16 scores and probabilities), 1 keeps them in fp32.
 *   scratch: device workspace of hyb_sdpa_decode_scratch_bytes() bytes, zeroed
 *   once before first use; the call leaves it ready for the next call.
 */
/*
 * The batch-1 qmv with the decode engine's fused prologue / epilogue (the
 * reference computes these as separate MLX ops: forward.cc:25-27 rms_norm,
 * :510-542 residual adds and layer_scalar, :324-343 GeGLU).
 *   prologue 0: x used as is; 1: x <- rms_norm(x, norm_w);
 *            2: h = bf16(resid + rms_norm(x, post_w)) [* scalar if non-NULL],
 *               h written to h_out (may be NULL), then x <- rms_norm(h, norm_w).
 *   epilogue 0: y[n] = bf16(x . w_hat[n]);
 *            1: rows are gate/up interleaved by 16-row tiles (tile 2t = gate rows
 *               16t..16t+15, tile 2t+1 = the matching up rows);
 *               y[n] = bf16(gelu_tanh(gate[n]) * up[n]) for n < N/2.
 *   x, resid, h_out, norm_w, post_w: bf16 [K]; scalar: bf16 [1].
 */
HypStatus hyb_qmv_fused(const void* x, const uint32_t* w, const void* scales, const void* biases,
                        void* y, int64_t K, int64_t N, int32_t prologue, int32_t epilogue,
                        const void* norm_w, const void* resid, const void* post_w,
                        const void* scalar, void* h_out, float eps, void* stream);

/*
 * Packed resident weight layout of the decode engine (no reference counterpart:
 * a load-time transform of the same MLX affine Q4/g64 tensors, like the
 * reference loader turning checkpoint tensors into its MLX arrays). Each 16-row x
 * 512-code block becomes one contiguous record in the order the qmv kernel's
 * tensor-core lanes consume it, with its scales and biases appended, so the
 * kernel streams every block with a single TMA bulk copy.
 *   hyb_qmv_packed_bytes: size of the packed form of an [N, K] matrix.
 *   hyb_qmv_pack: repack w/scales/biases (MLX layout) into `packed` (device,
 *   16-byte aligned). The MLX tensors may be freed afterwards.
 *   hyb_qmv_packed: the batch-1 qmv (with the hyb_qmv_fused prologue/epilogue
 *   options) reading the packed form; same results as hyb_qmv_fused.
 *   hyb_qmv_unpack: the inverse of hyb_qmv_pack (the engine's prefill GEMM
 *   re-derives each projection's MLX layout with it: the packed form is the only
 *   resident copy of the weights).
 *   hyb_embed_packed: embedding rows ids[0..L) of a packed [N, H] table,
 *   dequantised to bf16 and multiplied by embed_scale (bf16 bits), written to
 *   out [L][H]; ids must be < N (not checked on the device).
 */
size_t hyb_qmv_packed_bytes(int64_t K, int64_t N);
HypStatus hyb_qmv_pack(const uint32_t* w, const void* scales, const void* biases, int64_t K,
                       int64_t N, void* packed, void* stream);
HypStatus hyb_qmv_unpack(const void* packed, int64_t K, int64_t N, uint32_t* w, void* scales,
                         void* biases, void* stream);
HypStatus hyb_embed_packed(const uint32_t* ids, int64_t L, const void* packed, int64_t H, int64_t N,
                           uint16_t embed_scale_bf16, void* out, void* stream);
HypStatus hyb_qmv_packed(const void* x, const void* packed, void* y, int64_t K, int64_t N,
                         int32_t prologue, int32_t epilogue, const void* norm_w,
                         const void* resid, const void* post_w, const void* scalar,
                         void* h_out, float eps, void* stream);

size_t hyb_sdpa_decode_scratch_bytes(int32_t n_heads, int32_t n_kv, int32_t head_dim, int32_t max_keys);
HypStatus hyb_sdpa_decode(const void* q, const void* k_cache, const void* v_cache, void* out,
                          int32_t n_heads, int32_t n_kv, int32_t head_dim, int32_t capacity,
                          int32_t last_pos, int32_t n_keys, float scale, float softcap,
                          int32_t rounding, void* scratch, size_t scratch_bytes, void* stream);

/*
 * hyb_sdpa_decode without caller-provided scratch. This entry point has no
 * counterpart in the reference; it exists for callers that cannot call
 * cudaMalloc: a host runtime that hands the whole device to its own memory pool
 * and gives plugins no allocator, or a per-token loop that cannot afford the
 * device-wide synchronization a cudaMalloc may cause. It allocates nothing: its
 * scratch is a fixed 8 MiB (8388608-byte) array in device memory that every GPU
 * which loads this library holds until the process exits.
 *   Arguments, semantics and results are those of hyb_sdpa_decode.
 *   Limit: a call whose hyb_sdpa_decode_scratch_bytes(n_heads, n_kv, head_dim,
 *   n_keys) exceeds 8 MiB returns INVALID_ARGUMENT with a message naming the
 *   bytes it would need (e.g. 16 heads, 8 KV heads, head_dim 256 fit up to
 *   ~114k keys; the kernel itself accepts at most 32768).
 *   The first call on a device looks up the array's device address with that
 *   device current and caches it; make that first call before any stream capture.
 *   A caller that resets the device (cudaDeviceReset) must not call this entry
 *   point afterwards in the same process: the cached address would be stale.
 *   A rejected call (bad shape or a request above 8 MiB) queues no GPU work.
 *   All calls share the one array: it keeps the previous call's contents (each
 *   call clears the parts that must start at zero), and calls that overlap on the
 *   GPU (different streams, other threads) race with each other.
 */
HypStatus hyb_sdpa_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out,
                                  int32_t n_heads, int32_t n_kv, int32_t head_dim, int32_t capacity,
                                  int32_t last_pos, int32_t n_keys, float scale, float softcap,
                                  int32_t rounding, void* stream);

/*
 * The decode engine's fused single-token attention step, replacing for q_len == 1
 * the sequence q/k/v norms + RoPE + cache append + cache read + SDPA of
 * ForwardPass::attention (native/hyperion_mlx/src/forward.cc:394-504).
 *   qkv: bf16 raw projection row of the token: q (n_heads * head_dim), k (n_kv *
 *   head_dim), then v (n_kv * head_dim) unless v_from_k (global K=V layers: v is
 *   the weightless norm of the k columns). q and k are RMS-normalised with
 *   q_norm / k_norm [head_dim] and rotated at position pos with inv_freq
 *   [head_dim/2]; the new k and v are written to k_cache / v_cache
 *   [capacity, n_kv, head_dim] at slot pos % capacity; the query attends to the
 *   n_keys positions pos - n_keys + 1 .. pos. out: bf16 [n_heads, head_dim].
 *   Same score/probability rounding modes as hyb_sdpa_decode; no scratch. The
 *   n_keys scores live in the cluster's shared memory (about 200K keys for
 *   head_dim 256 and 2 query heads per KV head); longer contexts return
 *   INVALID_ARGUMENT (the engine then uses hyb_qkv_post + hyb_sdpa_decode).
 */
HypStatus hyb_sdpa_decode_fused(const void* qkv, int32_t v_from_k, const void* q_norm,
                                const void* k_norm, const float* inv_freq, float eps,
                                void* k_cache, void* v_cache, int32_t capacity, int32_t pos,
                                int32_t n_keys, int32_t n_heads, int32_t n_kv, int32_t head_dim,
                                float scale, float softcap, int32_t rounding, void* out,
                                void* stream);

/*
 * Tensor parallelism over TP GPUs of one node, one process per GPU (no reference
 * counterpart: the reference engine is single-device). Rank 0 creates a 128-byte NCCL
 * unique id and shares it with the other ranks by any host channel; every rank then
 * calls hyb_model_set_tensor_parallel on a created, not yet loaded model and loads it
 * (hyb_model_load_synthetic) at the same time, on its own current device. Each rank holds
 * its query/KV heads, 1/TP of the MLP and 1/TP of the vocabulary; o_proj and down_proj
 * partial sums are combined with an NCCL all-reduce, the greedy candidates with an
 * all-gather, and every rank returns the same tokens. Heads, KV heads, MLP rows (in
 * 16-row tiles and 64-wide groups) and the vocabulary must split evenly.
 */
HypStatus hyb_nccl_unique_id(void* out128);
HypStatus hyb_model_set_tensor_parallel(HypModel model, int32_t rank, int32_t size,
                                        const void* unique_id);

/*
 * Count of bounded shared-memory waits (mbarrier, bulk-copy completion) that gave
 * up on the current device since the library was loaded, summed over the
 * streaming qmv, the fused decode attention and the tensor-core prefill qmm. A wait that gives up leaves that
 * launch's output undefined but never hangs the GPU; the count is expected to stay
 * 0. No reference counterpart (the reference's kernels are MLX's).
 */
HypStatus hyb_wait_timeouts(int64_t* count);

/*
 * Multi-token causal attention with an optional sliding window, the prefill case
 * of the same op with the mask of build_mask (forward.cc:345-374).
 *   q: bf16 [Lq, n_heads, head_dim] at absolute positions q_pos0 + i;
 *   k, v: bf16 [Lk, n_kv, head_dim] at positions k_pos0 + j;
 *   key j is visible to query i iff kpos <= qpos and (window == 0 || kpos > qpos - window).
 *   out: bf16 [Lq, n_heads, head_dim].
 */
HypStatus hyb_sdpa_prefill(const void* q, const void* k, const void* v, void* out, int32_t Lq,
                           int32_t Lk, int32_t n_heads, int32_t n_kv, int32_t head_dim,
                           int32_t q_pos0, int32_t k_pos0, int32_t window, float scale,
                           float softcap, int32_t rounding, void* stream);

/*
 * Result of one device sampling call (hyb_sample_logits), written to device memory.
 */
typedef struct HybSampleResult {
    uint32_t token;             /* the sampled vocabulary index */
    float logit;                /* its post-softcap logit */
    uint32_t top_k_ids[8];      /* the 8 largest logits, value descending, index ascending */
    float top_k_values[8];
    uint32_t top_k_count;       /* min(8, n) */
    uint32_t kept;              /* tokens the top-p / min-p / top-k filters kept */
    float u;                    /* the uniform draw in [0, total) */
    float total;                /* the kept tokens' softmax weight sum (relative to the max) */
} HybSampleResult;

/*
 * Seeded stochastic sampling of one post-softcap bf16 logit row of length n on the
 * device, the step the sampled ABI calls run after their lm_head (replaces the host
 * sampler of native/hyperion_mlx/src/forward.cc:191-322 with its step order:
 * temperature, top-p, min-p, top-k, softmax, a draw u = uniform_real_distribution<float>
 * (0, total) from std::mt19937_64(rng_state), the first index whose running sum reaches
 * u). config follows hyp_decode_block_sampled's validation; temperature must be > 0.
 * `result` is device memory of sizeof(HybSampleResult) bytes. Among equal logits the
 * filters keep lower indices first. No device memory is allocated.
 */
HypStatus hyb_sample_logits(const void* logits, int32_t n, const HypSamplingConfig* config, uint64_t rng_state,
                            void* result, void* stream);

/*
 * RMSNorm over rows of length D: out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w);
 * w may be NULL (the weightless v_norm). Replaces mx::fast::rms_norm
 * (native/hyperion_mlx/src/forward.cc:25-27).
 */
HypStatus hyb_rms_norm(const void* x, const void* w, void* out, int32_t rows, int32_t D,
                       float eps, void* stream);

/*
 * QK-norm + RoPE + cache write for L tokens of one layer (forward.cc:394-420,
 * rope.cc:62-123, kv_cache.cc:161-249). qkv: bf16 [L, ld] holding q (n_heads * hd
 * columns), k (n_kv * hd), then v (n_kv * hd) unless v_from_k (global K=V layers:
 * V = v_norm of the k columns). inv_freq: f32 [hd/2] per-pair inverse frequencies
 * (0 = identity pair). Outputs: q_out [L, n_heads, hd]; k_out/v_out (optional)
 * [L, n_kv, hd]; k_cache/v_cache (optional) [cap, n_kv, hd] with slot (pos0+l) % cap
 * for tokens l >= cache_first.
 */
HypStatus hyb_qkv_post(const void* qkv, int32_t L, int32_t ld, int32_t n_heads, int32_t n_kv,
                       int32_t head_dim, int32_t v_from_k, const void* q_norm, const void* k_norm,
                       const float* inv_freq, int32_t pos0, float eps, void* q_out, void* k_out,
                       void* v_out, void* k_cache, void* v_cache, int32_t cache_cap,
                       int32_t cache_first, void* stream);

/*
 * Load seeded synthetic weights generated on the device (no checkpoint files),
 * for benchmarks at full model size. Every projection gets codes U{0..15},
 * scales bf16(|N(0, 0.02)|), biases -8 * scales; norms and layer_scalar
 * bf16(1 + N(0, 0.02)). Same validation and errors as hyp_model_load.
 */
HypStatus hyb_model_load_synthetic(HypModel model, const HypGeometryParams* geometry, uint64_t seed);

/*
 * Attention rounding of a loaded model: 0 (default) rounds scores and softmax
 * probabilities to bf16 as MLX's CPU-stream SDPA does (the semantics the parity
 * oracle follows); 1 keeps them in fp32 as MLX's fused Metal decode kernel does.
 */
HypStatus hyb_model_set_attention_rounding(HypModel model, int32_t mode);

/*
 * Batched decode qmv: y[b] = x[b] · Wᵀ for b < B (1..64) over packed weights
 * (hyb_qmv_pack), one weight stream for the batch. x is bf16 [B][ldx], y bf16 [B][ldy];
 * geglu != 0 applies the GeGLU epilogue of the interleaved gate/up matrix (N/2 outputs).
 * The codes are dequantised to fp16 (s·q + b, exact when b = −8s) and multiplied with
 * fp16 activations on the tensor cores in fp32.
 */
HypStatus hyb_qmv_batched(const void* x, int32_t B, int64_t ldx, const void* packed, void* y, int64_t ldy, int64_t K,
                          int64_t N, int32_t geglu, void* stream);

/*
 * A new KV state holding a copy of src (caches, position, commit counts) whose next
 * input token is last_token (UINT32_MAX keeps src's). Free it with hyp_kvstate_free.
 */
HypStatus hyb_kvstate_clone(HypModel model, HypKvState src, uint32_t last_token, HypKvState* out);

/*
 * Batched decode: one greedy step of n (1..64) distinct, populated KV states of the same
 * model in a single pass over the weights. Each state advances by one token from its own
 * last token; tokens_out[i] (and, when logits_out is not NULL, logits_out[i], the
 * post-softcap logit of that token) receive state i's result. Same validation as
 * hyp_decode_block; a failure after the step starts poisons every state of the batch.
 */
HypStatus hyb_decode_batch(HypModel model, const HypKvState* kvstates, uint32_t n, uint32_t* tokens_out,
                           float* logits_out);

/*
 * Greedy speculative verify of n_draft (1..8) draft tokens on a populated KV state: one
 * forward pass over [the state's last token, draft[0..n_draft)] at consecutive positions.
 * tokens_out[i] (n_draft + 1 entries) receives the greedy sample after input i, and
 * logits_out[i] (when not NULL) its post-softcap logit. The longest prefix of draft that
 * equals tokens_out is accepted (*n_accepted): the state advances by n_accepted + 1
 * tokens and its next input is tokens_out[n_accepted], so the outcome equals that many
 * greedy hyp_decode_block steps. The rejected tail stays in the local rings' speculative
 * slack (capacity window + 8) and is overwritten later; committed tokens are never
 * touched (kv.h:7-18). A failure after the pass starts poisons the state.
 */
HypStatus hyb_verify(HypModel model, HypKvState kv, const uint32_t* draft, uint32_t n_draft, uint32_t* tokens_out,
                     float* logits_out, uint32_t* n_accepted);

/* The CUDA stream the model's kernels run on (for event timing). */
HypStatus hyb_model_stream(HypModel model, void** out_stream);

/*
 * Copy a KV cache of layer `layer` to host memory for inspection: which = 0 for
 * K, 1 for V. Writes min(capacity rows, *rows) rows of n_kv * head_dim bf16 and
 * stores the cache capacity (ring capacity or global capacity) in *rows.
 */
HypStatus hyb_kv_copy_layer(HypModel model, HypKvState kv, uint32_t layer, int32_t which,
                            void* host_out, uint32_t* rows);

/* Current autoregressive cursor of a KV state (offset and last token). */
HypStatus hyb_kv_cursor(HypKvState kv, uint32_t* offset, uint32_t* last_token);

/*
 * Greedy steps that also copy the post-softcap logits (bf16, vocab entries,
 * host memory) of the step to `host_logits` (may be NULL). prefill uses
 * `tokens`; decode runs one step.
 */
HypStatus hyb_prefill_logits(HypModel model, HypKvState kv, const HypTokenStream* tokens,
                             HypStepResult out_result, void* host_logits);
HypStatus hyb_decode_logits(HypModel model, HypKvState kv, HypStepResult out_result,
                            void* host_logits);

/*
 * Decode with the next input token supplied by the caller instead of the last
 * sampled one (teacher forcing; used to measure per-step agreement without
 * divergence cascades).
 */
HypStatus hyb_decode_forced(HypModel model, HypKvState kv, uint32_t token, HypStepResult out_result,
                            void* host_logits);

/*
 * Test hook: the next prefill or decode call on this thread throws once on the
 * host right after its first forward has been enqueued, like the reference's
 * post-append fault (native/hyperion_mlx/src/test_fault.cc:1-24). The call
 * returns INTERNAL. A call that grew a global cache ran staged and is rolled
 * back (the state keeps its cursor and stays usable); any other call leaves the
 * KV state poisoned. No device fault is involved.
 */
HypStatus hyb_test_arm_post_append_fault(void);

/*
 * Memory budget of a loaded model: the ceiling, in device bytes held by the
 * engine (weights, KV caches, workspaces), that the predictive admission of
 * every prefill/decode call checks before doing any work (replaces the
 * platform-derived budget of the reference governor, governor.h:148-186).
 * A call whose predicted transient (staged global-cache growth, ring backups,
 * new workspace) would take the engine above it returns OOM_GOVERNOR with the
 * step result's governor_state = HYP_GOVERNOR_HARD_REJECT, and leaves the KV
 * state and its cursor untouched. 0 (the default) checks device free memory only.
 */
HypStatus hyb_model_set_memory_budget(HypModel model, uint64_t bytes);

/*
 * Weight memory of a loaded model (no reference counterpart: the reference holds
 * MLX arrays). resident = device bytes of the weights this rank holds: every
 * quantised matrix once, in the packed decode layout, plus norms and RoPE tables.
 * algorithmic = codes + scales + biases of those matrices (N*K/2 + N*K/16 bytes
 * each). scratch = the transient MLX-layout buffer the tensor-core prefill GEMM
 * re-derives one projection (or one lm_head slice) into. Any pointer may be NULL.
 */
HypStatus hyb_model_weight_bytes(HypModel model, uint64_t* resident, uint64_t* algorithmic, uint64_t* scratch);


#ifdef __cplusplus
}
#endif

#endif /* HYPERION_B200_H */
