// Op-level C entry points (include/hyperion_b200.h): each hot-path kernel behind
// plain pointers, sizes and a stream, with the library's status/error contract.
#include "hyperion_b200.h"
#include "kernels.h"

#include <cmath>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <exception>
#include <string>

namespace hyb {
HypStatus abi_fail(HypStatus s, const char* msg) noexcept;
HypStatus abi_ok() noexcept;
}  // namespace hyb

namespace {

template <typename Fn>
HypStatus run(Fn&& fn) noexcept {
    try {
        fn();
        return hyb::abi_ok();
    } catch (const hyb::ArgError& e) {
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, e.what());
    } catch (const hyb::CudaError& e) {
        return hyb::abi_fail(HYP_STATUS_INTERNAL, e.what());
    } catch (const std::exception& e) {
        return hyb::abi_fail(HYP_STATUS_INTERNAL, e.what());
    } catch (...) {
        return hyb::abi_fail(HYP_STATUS_INTERNAL, "op failed with a non-standard exception");
    }
}

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

HypStatus hyb_build_info(char* buffer, size_t len) {
    if (buffer == nullptr || len == 0) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "buffer is null");
    std::snprintf(buffer, len, "hyperion_b200 sm_100a cuda %d", CUDART_VERSION);
    return hyb::abi_ok();
}

HypStatus hyb_quantized_matmul(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                               int64_t M, int64_t K, int64_t N, int32_t group_size, int32_t bits, void* stream) {
    if (group_size != 64 || bits != 4)
        return hyb::abi_fail(HYP_STATUS_UNSUPPORTED, "only affine group_size=64, bits=4 is implemented");
    if (!x || !w || !scales || !biases || !y) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (M <= 0 || N <= 0 || K <= 0 || K % 64 != 0 || M > (1 << 24) || N > (1 << 30) || K > (1 << 20))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "quantized_matmul: bad shape (K must be a positive multiple of 64)");
    if (!aligned16(x) || !aligned16(w) || !aligned16(y))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "quantized_matmul: x, w and y must be 16-byte aligned");
    return run([&] {
        hyb::launch_quantized_matmul(static_cast<const hyb::bf16*>(x), w, static_cast<const hyb::bf16*>(scales),
                                     static_cast<const hyb::bf16*>(biases), static_cast<hyb::bf16*>(y),
                                     static_cast<int>(M), static_cast<int>(K), static_cast<int>(N), as_stream(stream));
    });
}

HypStatus hyb_qmv_fused(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                        int64_t K, int64_t N, int32_t prologue, int32_t epilogue, const void* norm_w,
                        const void* resid, const void* post_w, const void* scalar, void* h_out, float eps,
                        void* stream) {
    if (!x || !w || !scales || !biases || !y) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (K <= 0 || K % 64 != 0 || N <= 0 || K > (1 << 20) || N > (1 << 30))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_fused: bad shape");
    if (prologue < 0 || prologue > 2 || epilogue < 0 || epilogue > 1)
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_fused: unknown prologue/epilogue");
    if (prologue >= 1 && !norm_w) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_fused: norm_w is required");
    if (prologue == 2 && (!resid || !post_w)) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_fused: resid and post_w are required");
    if (epilogue == 1 && N % 32 != 0) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_fused: GeGLU rows must be a multiple of 32");
    if (prologue != 0 && K * 4 > 96 * 1024) return hyb::abi_fail(HYP_STATUS_UNSUPPORTED, "qmv_fused: K too large for a norm prologue");
    return run([&] {
        hyb::QmvParams p;
        p.x = static_cast<const hyb::bf16*>(x);
        p.w = w;
        p.s = static_cast<const hyb::bf16*>(scales);
        p.b = static_cast<const hyb::bf16*>(biases);
        p.y = static_cast<hyb::bf16*>(y);
        p.K = static_cast<int>(K);
        p.N = static_cast<int>(N);
        p.prologue = static_cast<hyb::QmvPrologue>(prologue);
        p.epilogue = static_cast<hyb::QmvEpilogue>(epilogue);
        p.norm_w = static_cast<const hyb::bf16*>(norm_w);
        p.resid = static_cast<const hyb::bf16*>(resid);
        p.post_w = static_cast<const hyb::bf16*>(post_w);
        p.scalar = static_cast<const hyb::bf16*>(scalar);
        p.h_out = static_cast<hyb::bf16*>(h_out);
        p.eps = eps;
        hyb::launch_qmv(p, as_stream(stream), false);
    });
}

size_t hyb_qmv_packed_bytes(int64_t K, int64_t N) {
    if (K <= 0 || K % 64 != 0 || N <= 0 || K > (1 << 20) || N > (1 << 30)) return 0;
    return hyb::qmv_packed_bytes(static_cast<int>(K), static_cast<int>(N));
}

HypStatus hyb_qmv_pack(const uint32_t* w, const void* scales, const void* biases, int64_t K, int64_t N, void* packed,
                       void* stream) {
    if (!w || !scales || !biases || !packed) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (K <= 0 || K % 64 != 0 || N <= 0 || K > (1 << 20) || N > (1 << 30))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_pack: bad shape");
    if (!aligned16(w) || !aligned16(packed)) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_pack: w and packed must be 16-byte aligned");
    return run([&] {
        hyb::launch_qmv_pack(w, static_cast<const hyb::bf16*>(scales), static_cast<const hyb::bf16*>(biases),
                             static_cast<int>(K), static_cast<int>(N), packed, as_stream(stream));
    });
}

HypStatus hyb_qmv_unpack(const void* packed, int64_t K, int64_t N, uint32_t* w, void* scales, void* biases,
                         void* stream) {
    if (!w || !scales || !biases || !packed) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (K <= 0 || K % 64 != 0 || N <= 0 || K > (1 << 20) || N > (1 << 30))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_unpack: bad shape");
    if (!aligned16(w) || !aligned16(packed)) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_unpack: w and packed must be 16-byte aligned");
    return run([&] {
        hyb::launch_qmv_unpack(packed, static_cast<int>(K), static_cast<int>(N), w, static_cast<hyb::bf16*>(scales),
                               static_cast<hyb::bf16*>(biases), as_stream(stream));
    });
}

HypStatus hyb_embed_packed(const uint32_t* ids, int64_t L, const void* packed, int64_t H, int64_t N,
                           uint16_t embed_scale_bf16, void* out, void* stream) {
    if (!ids || !packed || !out) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (L <= 0 || L > 65535 || H <= 0 || H % 64 != 0 || H > (1 << 20) || N <= 0 || N > (1 << 30))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "embed_packed: bad shape");
    if (!aligned16(packed) || !aligned16(out)) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "embed_packed: packed and out must be 16-byte aligned");
    hyb::bf16 sc;
    std::memcpy(&sc, &embed_scale_bf16, 2);
    return run([&] {
        hyb::launch_embed_packed(ids, static_cast<int>(L), packed, static_cast<int>(H), static_cast<int>(N), sc,
                                 static_cast<hyb::bf16*>(out), as_stream(stream));
    });
}

HypStatus hyb_qmv_packed(const void* x, const void* packed, void* y, int64_t K, int64_t N, int32_t prologue,
                         int32_t epilogue, const void* norm_w, const void* resid, const void* post_w,
                         const void* scalar, void* h_out, float eps, void* stream) {
    if (!x || !packed || !y) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (K <= 0 || K % 64 != 0 || N <= 0 || K > (1 << 20) || N > (1 << 30))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_packed: bad shape");
    if (prologue < 0 || prologue > 2 || epilogue < 0 || epilogue > 1)
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_packed: unknown prologue/epilogue");
    if (prologue >= 1 && !norm_w) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_packed: norm_w is required");
    if (prologue == 2 && (!resid || !post_w)) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_packed: resid and post_w are required");
    if (epilogue == 1 && N % 32 != 0) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_packed: GeGLU rows must be a multiple of 32");
    return run([&] {
        hyb::QmvParams p;
        p.x = static_cast<const hyb::bf16*>(x);
        p.packed = packed;
        p.y = static_cast<hyb::bf16*>(y);
        p.K = static_cast<int>(K);
        p.N = static_cast<int>(N);
        p.prologue = static_cast<hyb::QmvPrologue>(prologue);
        p.epilogue = static_cast<hyb::QmvEpilogue>(epilogue);
        p.norm_w = static_cast<const hyb::bf16*>(norm_w);
        p.resid = static_cast<const hyb::bf16*>(resid);
        p.post_w = static_cast<const hyb::bf16*>(post_w);
        p.scalar = static_cast<const hyb::bf16*>(scalar);
        p.h_out = static_cast<hyb::bf16*>(h_out);
        p.eps = eps;
        hyb::launch_qmv_packed(p, as_stream(stream), true);
    });
}

HypStatus hyb_qmv_batched(const void* x, int32_t B, int64_t ldx, const void* packed, void* y, int64_t ldy, int64_t K,
                          int64_t N, int32_t geglu, void* stream) {
    if (!x || !packed || !y) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (B < 1 || B > hyb::kMaxDecodeBatch) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_batched: batch must be 1..64");
    if (K <= 0 || K % 64 != 0 || N <= 0 || K > (1 << 20) || N > (1 << 30) || ldx < K || ldy < (geglu ? N / 2 : N))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_batched: bad shape");
    if (geglu && N % 32 != 0) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qmv_batched: GeGLU rows must be a multiple of 32");
    return run([&] {
        cudaStream_t st = as_stream(stream);
        void* x16 = nullptr;
        HYB_CUDA(cudaMallocAsync(&x16, hyb::qmv_batch_x16_words(B, static_cast<int>(K)) * 4, st));
        hyb::launch_qmv_batched_x16(static_cast<const hyb::bf16*>(x), B, static_cast<int>(ldx), static_cast<int>(K),
                                    static_cast<uint32_t*>(x16), st);
        hyb::QmvBatchParams q;
        q.x16 = static_cast<const uint32_t*>(x16);
        q.packed = packed;
        q.y = static_cast<hyb::bf16*>(y);
        q.K = static_cast<int>(K);
        q.N = static_cast<int>(N);
        q.B = B;
        q.ldy = static_cast<int>(ldy);
        q.geglu = geglu != 0;
        hyb::launch_qmv_batched(q, st);
        HYB_CUDA(cudaFreeAsync(x16, st));
    });
}

size_t hyb_sdpa_decode_scratch_bytes(int32_t n_heads, int32_t n_kv, int32_t head_dim, int32_t max_keys) {
    if (n_heads <= 0 || n_kv <= 0 || head_dim <= 0 || max_keys <= 0) return 0;
    return hyb::decode_attn_scratch_bytes(n_heads, n_kv, head_dim, max_keys);
}

HypStatus hyb_sdpa_decode(const void* q, const void* k_cache, const void* v_cache, void* out, int32_t n_heads,
                          int32_t n_kv, int32_t head_dim, int32_t capacity, int32_t last_pos, int32_t n_keys,
                          float scale, float softcap, int32_t rounding, void* scratch, size_t scratch_bytes,
                          void* stream) {
    if (!q || !k_cache || !v_cache || !out || !scratch)
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0 || n_keys <= 0 || capacity <= 0 || last_pos < n_keys - 1)
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sdpa_decode: bad shape");
    if (n_keys > capacity) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sdpa_decode: n_keys exceeds the cache capacity");
    if (head_dim != 64 && head_dim != 128 && head_dim != 256 && head_dim != 512)
        return hyb::abi_fail(HYP_STATUS_UNSUPPORTED, "sdpa_decode: head_dim must be 64, 128, 256 or 512");
    return run([&] {
        hyb::DecodeAttnParams p;
        p.q = static_cast<const hyb::bf16*>(q);
        p.k_cache = static_cast<const hyb::bf16*>(k_cache);
        p.v_cache = static_cast<const hyb::bf16*>(v_cache);
        p.out = static_cast<hyb::bf16*>(out);
        p.n_heads = n_heads;
        p.n_kv = n_kv;
        p.hd = head_dim;
        p.cap = capacity;
        p.last_pos = last_pos;
        p.n_keys = n_keys;
        p.scale = scale;
        p.softcap = softcap;
        p.rounding = rounding;
        p.scratch = scratch;
        p.scratch_bytes = scratch_bytes;
        hyb::launch_decode_attn(p, as_stream(stream));
    });
}

HypStatus hyb_sdpa_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out,
                                  int32_t n_heads, int32_t n_kv, int32_t head_dim, int32_t capacity,
                                  int32_t last_pos, int32_t n_keys, float scale, float softcap, int32_t rounding,
                                  void* stream) {
    if (!q || !k_cache || !v_cache || !out) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0 || n_keys <= 0 || capacity <= 0 || last_pos < n_keys - 1)
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sdpa_decode_noalloc: bad shape");
    if (n_keys > capacity)
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sdpa_decode_noalloc: n_keys exceeds the cache capacity");
    if (head_dim != 64 && head_dim != 128 && head_dim != 256 && head_dim != 512)
        return hyb::abi_fail(HYP_STATUS_UNSUPPORTED, "sdpa_decode_noalloc: head_dim must be 64, 128, 256 or 512");
    return run([&] {
        hyb::DecodeAttnParams p;
        p.q = static_cast<const hyb::bf16*>(q);
        p.k_cache = static_cast<const hyb::bf16*>(k_cache);
        p.v_cache = static_cast<const hyb::bf16*>(v_cache);
        p.out = static_cast<hyb::bf16*>(out);
        p.n_heads = n_heads;
        p.n_kv = n_kv;
        p.hd = head_dim;
        p.cap = capacity;
        p.last_pos = last_pos;
        p.n_keys = n_keys;
        p.scale = scale;
        p.softcap = softcap;
        p.rounding = rounding;
        hyb::launch_decode_attn_noalloc(p, as_stream(stream));
    });
}

HypStatus hyb_sdpa_decode_fused(const void* qkv, int32_t v_from_k, const void* q_norm, const void* k_norm,
                                const float* inv_freq, float eps, void* k_cache, void* v_cache, int32_t capacity,
                                int32_t pos, int32_t n_keys, int32_t n_heads, int32_t n_kv, int32_t head_dim,
                                float scale, float softcap, int32_t rounding, void* out, void* stream) {
    if (!qkv || !q_norm || !k_norm || !inv_freq || !k_cache || !v_cache || !out)
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0 || n_keys <= 0 || capacity < n_keys || pos < n_keys - 1)
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sdpa_decode_fused: bad shape");
    if (head_dim != 64 && head_dim != 128 && head_dim != 256)
        return hyb::abi_fail(HYP_STATUS_UNSUPPORTED, "sdpa_decode_fused: head_dim must be 64, 128 or 256");
    return run([&] {
        hyb::DecodeFusedParams p;
        p.qkv = static_cast<const hyb::bf16*>(qkv);
        p.v_from_k = v_from_k != 0;
        p.q_norm = static_cast<const hyb::bf16*>(q_norm);
        p.k_norm = static_cast<const hyb::bf16*>(k_norm);
        p.inv_freq = inv_freq;
        p.eps = eps;
        p.k_cache = static_cast<hyb::bf16*>(k_cache);
        p.v_cache = static_cast<hyb::bf16*>(v_cache);
        p.cap = capacity;
        p.pos = pos;
        p.n_keys = n_keys;
        p.n_heads = n_heads;
        p.n_kv = n_kv;
        p.hd = head_dim;
        p.scale = scale;
        p.softcap = softcap;
        p.rounding = rounding;
        p.out = static_cast<hyb::bf16*>(out);
        hyb::launch_decode_attn_fused(p, as_stream(stream), false);
    });
}

HypStatus hyb_sdpa_prefill(const void* q, const void* k, const void* v, void* out, int32_t Lq, int32_t Lk,
                           int32_t n_heads, int32_t n_kv, int32_t head_dim, int32_t q_pos0, int32_t k_pos0,
                           int32_t window, float scale, float softcap, int32_t rounding, void* stream) {
    if (!q || !k || !v || !out) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (Lq <= 0 || Lk <= 0 || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0 || window < 0)
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sdpa_prefill: bad shape");
    if (head_dim != 64 && head_dim != 128 && head_dim != 256)
        return hyb::abi_fail(HYP_STATUS_UNSUPPORTED, "sdpa_prefill: head_dim must be 64, 128 or 256");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sdpa_prefill: q, k, v must be 16-byte aligned");
    return run([&] {
        hyb::PrefillAttnParams p;
        p.q = static_cast<const hyb::bf16*>(q);
        p.k = static_cast<const hyb::bf16*>(k);
        p.v = static_cast<const hyb::bf16*>(v);
        p.out = static_cast<hyb::bf16*>(out);
        p.Lq = Lq;
        p.Lk = Lk;
        p.n_heads = n_heads;
        p.n_kv = n_kv;
        p.hd = head_dim;
        p.q_pos0 = q_pos0;
        p.k_pos0 = k_pos0;
        p.window = window;
        p.scale = scale;
        p.softcap = softcap;
        p.rounding = rounding;
        hyb::launch_prefill_attn(p, as_stream(stream));
    });
}

static_assert(sizeof(HybSampleResult) == sizeof(hyb::SampleResult), "HybSampleResult mirrors hyb::SampleResult");
static_assert(offsetof(HybSampleResult, top_k_count) == offsetof(hyb::SampleResult, topk_count),
              "HybSampleResult mirrors hyb::SampleResult");

HypStatus hyb_sample_logits(const void* logits, int32_t n, const HypSamplingConfig* config, uint64_t rng_state,
                            void* result, void* stream) {
    if (!logits || !config || !result) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (n <= 0) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sample_logits: empty row");
    if (!(config->temperature > 0.0f)) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sample_logits: temperature must be > 0");
    if (config->top_k < 0 || config->top_k > n) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sample_logits: top_k must be in [0, n]");
    if (!std::isnan(config->top_p) && (config->top_p < 0.0f || config->top_p > 1.0f))
        return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sample_logits: top_p must be in [0, 1]");
    if (config->min_p < 0.0f || config->min_p >= 1.0f) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "sample_logits: min_p must be in [0, 1)");
    return run([&] {
        hyb::SampleSpec sp;
        sp.temperature = config->temperature;
        sp.top_k = config->top_k;
        sp.top_p = std::isnan(config->top_p) ? 0.f : config->top_p;
        sp.min_p = config->min_p;
        sp.seed = rng_state;
        hyb::launch_sample(static_cast<const hyb::bf16*>(logits), n, sp, static_cast<hyb::SampleResult*>(result),
                           as_stream(stream));
    });
}

HypStatus hyb_rms_norm(const void* x, const void* w, void* out, int32_t rows, int32_t D, float eps, void* stream) {
    if (!x || !out) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (rows < 0 || D <= 0) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "rms_norm: bad shape");
    return run([&] {
        hyb::launch_rms_norm(static_cast<const hyb::bf16*>(x), static_cast<const hyb::bf16*>(w),
                             static_cast<hyb::bf16*>(out), rows, D, eps, as_stream(stream));
    });
}

HypStatus hyb_qkv_post(const void* qkv, int32_t L, int32_t ld, int32_t n_heads, int32_t n_kv, int32_t head_dim,
                       int32_t v_from_k, const void* q_norm, const void* k_norm, const float* inv_freq, int32_t pos0,
                       float eps, void* q_out, void* k_out, void* v_out, void* k_cache, void* v_cache,
                       int32_t cache_cap, int32_t cache_first, void* stream) {
    if (!qkv || !q_norm || !k_norm || !inv_freq || !q_out) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "null pointer argument");
    if (L <= 0 || n_heads <= 0 || n_kv <= 0 || pos0 < 0) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qkv_post: bad shape");
    if (head_dim % 64 != 0 || head_dim > 512) return hyb::abi_fail(HYP_STATUS_UNSUPPORTED, "qkv_post: head_dim must be a multiple of 64 up to 512");
    const int64_t need = static_cast<int64_t>(n_heads + (v_from_k ? 1 : 2) * n_kv) * head_dim;
    if (ld < need) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qkv_post: ld smaller than the q/k/v columns");
    if ((k_cache || v_cache) && cache_cap <= 0) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "qkv_post: cache_cap must be positive");
    return run([&] {
        hyb::QkvPostParams p;
        p.qkv = static_cast<const hyb::bf16*>(qkv);
        p.L = L;
        p.ld = ld;
        p.n_heads = n_heads;
        p.n_kv = n_kv;
        p.hd = head_dim;
        p.v_from_k = v_from_k != 0;
        p.q_norm = static_cast<const hyb::bf16*>(q_norm);
        p.k_norm = static_cast<const hyb::bf16*>(k_norm);
        p.inv_freq = inv_freq;
        p.pos0 = pos0;
        p.eps = eps;
        p.q_out = static_cast<hyb::bf16*>(q_out);
        p.k_out = static_cast<hyb::bf16*>(k_out);
        p.v_out = static_cast<hyb::bf16*>(v_out);
        p.k_cache = static_cast<hyb::bf16*>(k_cache);
        p.v_cache = static_cast<hyb::bf16*>(v_cache);
        p.cache_cap = cache_cap;
        p.cache_first = cache_first;
        hyb::launch_qkv_post(p, as_stream(stream));
    });
}

HypStatus hyb_wait_timeouts(int64_t* count) {
    if (!count) return hyb::abi_fail(HYP_STATUS_INVALID_ARGUMENT, "count is null");
    return run([&] {
        *count = hyb::read_qmv_wait_timeouts() + hyb::read_qmvb_wait_timeouts() + hyb::read_attn_wait_timeouts() +
                 hyb::read_attn_tc_wait_timeouts() + hyb::read_qmm_wait_timeouts();
    });
}

}  // extern "C"
