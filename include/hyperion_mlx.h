/*
 * hyperion_mlx.h - the 14-function engine ABI, served by the B200 CUDA engine.
 *
 * This header declares the same C interface that Hyperion's Rust `hyperion-ffi`
 * crate binds (reference: native/hyperion_mlx/include/hyperion_mlx.h:1-254).
 * Type names, enumerator values, struct field order and function signatures are
 * kept identical so that the Rust side links against libhyperion_mlx built from
 * this repository without any change; only the implementation behind it differs
 * (hand-written sm_100a kernels instead of MLX/Metal).
 *
 * The header is plain C11 and must compile with -std=c11 -Wpedantic -Werror.
 */
#ifndef HYPERION_MLX_H
#define HYPERION_MLX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every function below (reference hyperion_mlx.h:12-21). */
typedef enum HypStatus {
    HYP_STATUS_OK = 0,
    HYP_STATUS_INVALID_ARGUMENT = 1,
    HYP_STATUS_NOT_FOUND = 2,
    HYP_STATUS_IO = 3,
    HYP_STATUS_OOM_GOVERNOR = 4,
    HYP_STATUS_UNSUPPORTED = 5,
    HYP_STATUS_INTERNAL = 6,
    HYP_STATUS_CANCELLED = 7
} HypStatus;

/*
 * Platform canary record (reference hyperion_mlx.h:24-41; sizeof == 224, with
 * recommended_working_set_bytes at offset 32, mlx_runtime_version at 64 and
 * gpu_name at 96). On the CUDA engine the "mlx_*" fields carry the CUDA runtime
 * version, the macOS fields carry the CUDA driver version, gpu_family carries the
 * SM version (100 for sm_100), and the byte budgets come from cudaMemGetInfo.
 */
typedef struct HypCanaryInfo {
    uint32_t abi_version;
    uint32_t mlx_compile_major;
    uint32_t mlx_compile_minor;
    uint32_t mlx_compile_patch;
    uint32_t macos_major;
    uint32_t macos_minor;
    uint32_t macos_patch;
    uint32_t gpu_family;
    uint64_t recommended_working_set_bytes;
    uint64_t effective_budget_bytes;
    uint64_t soft_watermark_bytes;
    float mlx_probe_value;
    float metallib_probe_value;
    char mlx_runtime_version[32];
    char gpu_name[128];
} HypCanaryInfo;

/* Probe the device and run two tiny kernels; fills *out_info. */
HypStatus hyp_runtime_canary(HypCanaryInfo* out_info);

/* Copy the calling thread's last error message (NUL-terminated, truncated). */
HypStatus hyp_last_error(char* buffer, size_t buffer_len);

/* Opaque, magic-tagged handles (reference hyperion_mlx.h:46-50). */
typedef struct HypModelOpaque* HypModel;
typedef struct HypKvStateOpaque* HypKvState;
typedef struct HypStepResultOpaque* HypStepResult;

typedef enum HypTextModelType {
    HYP_GEMMA4_TEXT = 0,
    HYP_GEMMA4_UNIFIED_TEXT = 1
} HypTextModelType;

typedef enum HypLayerType {
    HYP_LAYER_SLIDING = 0,
    HYP_LAYER_FULL = 1
} HypLayerType;

typedef enum HypGovernorState {
    HYP_GOVERNOR_READY = 0,
    HYP_GOVERNOR_SOFT_PAUSED = 1,
    HYP_GOVERNOR_HARD_REJECT = 2
} HypGovernorState;

/* RoPE parameters of one attention kind (reference hyperion_mlx.h:73-79). */
typedef struct HypRopeSpec {
    double theta;
    int has_partial_rotary_factor;
    float partial_rotary_factor;
    int proportional;
} HypRopeSpec;

typedef struct HypMoeConfig {
    uint32_t num_experts;
    uint32_t top_k;
    uint32_t moe_intermediate_size;
} HypMoeConfig;

/* Model geometry as validated by the Rust side (reference hyperion_mlx.h:89-116). */
typedef struct HypGeometryParams {
    HypTextModelType model_type;
    uint32_t hidden_size;
    uint32_t intermediate_size;
    uint32_t num_hidden_layers;
    const HypLayerType* layer_types;
    uint32_t num_attention_heads;
    uint32_t head_dim_local;
    uint32_t head_dim_global;
    uint32_t num_kv_heads_local;
    uint32_t num_kv_heads_global;
    int attention_k_eq_v_global;
    uint32_t num_kv_shared_layers;
    uint32_t sliding_window;
    HypRopeSpec rope_local;
    HypRopeSpec rope_global;
    float final_logit_softcapping;
    float rms_norm_eps;
    int attention_bias;
    uint32_t vocab_size;
    uint32_t max_position_embeddings;
    int tie_word_embeddings;
    uint32_t ple_hidden_per_layer_input;
    uint32_t ple_vocab_per_layer_input;
    int use_double_wide_mlp;
    int has_moe;
    HypMoeConfig moe;
} HypGeometryParams;

/* Token ids for prefill (is_prompt = 1) or decode (reference hyperion_mlx.h:119-123). */
typedef struct HypTokenStream {
    const uint32_t* tokens;
    uint32_t count;
    int is_prompt;
} HypTokenStream;

/*
 * Sampling configuration (reference hyperion_mlx.h:134-140). NULL or
 * temperature == 0 selects greedy argmax, bit-identical to the unsampled calls.
 */
typedef struct HypSamplingConfig {
    float temperature;
    int32_t top_k;
    float top_p;
    float min_p;
    uint64_t seed;
} HypSamplingConfig;

/* Size of the per-step top-k sidecar (reference hyperion_mlx.h:145). */
#define HYP_TOP_K_LOGPROBS 8

/*
 * Per-step result (reference hyperion_mlx.h:157-176). On the CUDA engine the
 * "*_mlx_bytes" fields report CUDA device-memory figures of this library's
 * allocations; local/global_kv_bytes are the allocated cache capacities.
 */
typedef struct {
    uint32_t token_id;
    float logit;
    uint64_t peak_mlx_bytes;
    uint64_t active_mlx_bytes;
    uint64_t phys_footprint_bytes;
    uint64_t local_kv_bytes;
    uint64_t global_kv_bytes;
    float local_kv_eval_ms;
    float global_kv_eval_ms;
    HypGovernorState governor_state;
    uint32_t near_tie_events;
    uint32_t top_k_logprob_count;
    uint32_t top_k_logprob_ids[HYP_TOP_K_LOGPROBS];
    float top_k_logprob_values[HYP_TOP_K_LOGPROBS];
} HypStepResultFields;

HypStatus hyp_model_create(HypModel* out_model);
HypStatus hyp_model_free(HypModel* model);

/* Validate geometry, read every *.safetensors under weights_path, pack to HBM. */
HypStatus hyp_model_load(HypModel model,
                         const HypGeometryParams* geometry,
                         const char* weights_path);

HypStatus hyp_kvstate_create(HypModel model, HypKvState* out_kvstate);
HypStatus hyp_kvstate_free(HypKvState* kvstate);

/* Prefill a whole prompt into a fresh KV state (chunks of 2048 internally). */
HypStatus hyp_prefill_chunk(HypModel model,
                            HypKvState kvstate,
                            const HypTokenStream* tokens,
                            HypStepResult out_result);

/* Greedy-decode n_tokens, each fed back as the next input. */
HypStatus hyp_decode_block(HypModel model,
                           HypKvState kvstate,
                           uint32_t n_tokens,
                           HypStepResult out_result);

HypStatus hyp_prefill_chunk_sampled(HypModel model,
                                    HypKvState kvstate,
                                    const HypTokenStream* tokens,
                                    const HypSamplingConfig* config,
                                    HypStepResult out_result);

HypStatus hyp_decode_block_sampled(HypModel model,
                                   HypKvState kvstate,
                                   uint32_t n_tokens,
                                   const HypSamplingConfig* config,
                                   HypStepResult out_result);

HypStatus hyp_step_result_create(HypStepResult* out_result);
HypStatus hyp_step_result_free(HypStepResult* result);
HypStatus hyp_step_result_fields(HypStepResult result,
                                 HypStepResultFields* out_fields);

#ifdef __cplusplus
}
#endif

#endif /* HYPERION_MLX_H */
