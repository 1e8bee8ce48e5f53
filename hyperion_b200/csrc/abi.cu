// The hyperion_mlx.h ABI over the CUDA engine, plus the hyperion_b200.h extensions.
//
// Handle, status and error semantics follow the reference ABI implementation
// (native/hyperion_mlx/src/model.cc:129-207 handles, :234-254 sampler-config
// validation, :361-995 entry points; runtime.mm:223-298 canary / last error;
// abi_error.cc thread-local message). No exception crosses the C boundary.
#include "engine.h"
#include "hyperion_b200.h"
#include "hyperion_mlx.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <limits>
#include <memory>
#include <new>
#include <optional>
#include <string>
#include <vector>

// Opaque handle bodies (global namespace to match the header's struct tags).
struct HypModelOpaque {
    uint32_t magic;
    bool loaded = false;
    std::unique_ptr<hyb::Model> model;
    int tp_rank = 0, tp_size = 1;       // tensor parallelism requested before the load
    unsigned char tp_id[128] = {};
};

struct HypKvStateOpaque {
    uint32_t magic;
    std::unique_ptr<hyb::KvState> kv;
    const HypModelOpaque* owner = nullptr;
};

struct HypStepResultOpaque {
    uint32_t magic;
    HypStepResultFields fields;
};

namespace {

constexpr uint32_t kModelMagic = 0x48504D4FU;       // "HPMO"
constexpr uint32_t kKvStateMagic = 0x48504B56U;     // "HPKV"
constexpr uint32_t kStepResultMagic = 0x48505352U;  // "HPSR"
constexpr uint32_t kAbiVersion = 3;
constexpr size_t kLastErrorCapacity = 1024;

thread_local char g_last_error[kLastErrorCapacity] = {0};
thread_local bool g_fault_armed = false;

HypStatus fail(HypStatus s, const char* msg) noexcept {
    std::snprintf(g_last_error, kLastErrorCapacity, "%s", msg ? msg : "unknown native error");
    return s;
}
HypStatus fail(HypStatus s, const std::string& msg) noexcept { return fail(s, msg.c_str()); }
HypStatus ok() noexcept {
    g_last_error[0] = '\0';
    return HYP_STATUS_OK;
}

}  // namespace

namespace hyb {
// Shared with the op-level entry points (ops_abi.cu).
HypStatus abi_fail(HypStatus s, const char* msg) noexcept { return fail(s, msg); }
HypStatus abi_ok() noexcept { return ok(); }
}  // namespace hyb

namespace {

HypStatus validate_model(HypModel m) noexcept {
    if (m == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "model handle is null");
    if (m->magic != kModelMagic)
        return fail(HYP_STATUS_INVALID_ARGUMENT, "model handle magic mismatch (wrong type, freed, or corrupted)");
    return ok();
}
HypStatus validate_kv(HypKvState kv) noexcept {
    if (kv == nullptr || kv->magic != kKvStateMagic) return fail(HYP_STATUS_INVALID_ARGUMENT, "kvstate handle is invalid");
    if (kv->kv && kv->kv->poisoned)
        return fail(HYP_STATUS_INTERNAL, "KV state is unusable after an internal execution failure; free and recreate it");
    return ok();
}
HypStatus validate_result(HypStepResult r) noexcept {
    if (r == nullptr || r->magic != kStepResultMagic) return fail(HYP_STATUS_INVALID_ARGUMENT, "step-result handle is invalid");
    return ok();
}

template <typename H>
HypStatus create_handle(H** out, uint32_t magic) noexcept {
    if (out == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "create requires a non-null out handle");
    try {
        auto* h = new H{};
        h->magic = magic;
        *out = h;
        return ok();
    } catch (const std::bad_alloc&) {
        return fail(HYP_STATUS_INTERNAL, "native allocation failed outside predictive governor admission");
    } catch (...) {
        return fail(HYP_STATUS_INTERNAL, "unexpected exception in handle create");
    }
}

template <typename H>
HypStatus free_handle(H** h, uint32_t magic) noexcept {
    if (h == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "free requires a non-null handle pointer");
    H* p = *h;
    if (p == nullptr) return ok();
    if (p->magic != magic) return fail(HYP_STATUS_INVALID_ARGUMENT, "handle magic mismatch (wrong type, freed, or corrupted)");
    p->magic = 0;
    try {
        delete p;
    } catch (...) {
    }
    *h = nullptr;
    return ok();
}

// Run `fn` mapping exceptions to statuses (model.cc:442-452).
template <typename Fn>
HypStatus guarded(const char* op, Fn&& fn) noexcept {
    try {
        return fn();
    } catch (const std::filesystem::filesystem_error& e) {
        return fail(HYP_STATUS_IO, e.what());
    } catch (const std::bad_alloc&) {
        return fail(HYP_STATUS_INTERNAL, "native allocation failed outside predictive governor admission");
    } catch (const std::exception& e) {
        return fail(HYP_STATUS_INTERNAL, e.what());
    } catch (...) {
        return fail(HYP_STATUS_INTERNAL, std::string(op) + " failed with a non-standard exception");
    }
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) hyb::cuda_check(cudaSetDevice(dev), "cudaSetDevice");
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

void write_result(HypStepResult r, const hyb::StepOut* s, uint32_t near_ties, HypGovernorState state,
                  const hyb::Model& m, const hyb::KvState& kv, bool sampled) {
    HypStepResultFields f{};
    if (s) {
        f.token_id = s->token;
        f.logit = s->logit;
        if (sampled) {
            const uint32_t n = std::min<uint32_t>(HYP_TOP_K_LOGPROBS, m.geometry().vocab);
            f.top_k_logprob_count = n;
            for (uint32_t i = 0; i < n; ++i) {
                f.top_k_logprob_ids[i] = s->topk_idx[i];
                f.top_k_logprob_values[i] = s->topk_val[i];
            }
        }
    }
    f.peak_mlx_bytes = hyb::dev_peak_bytes();
    f.active_mlx_bytes = hyb::dev_active_bytes();
    f.local_kv_bytes = m.local_kv_bytes(kv);
    f.global_kv_bytes = m.global_kv_bytes(kv);
    f.governor_state = state;
    f.near_tie_events = sampled ? 0u : near_ties;
    r->fields = f;
}

std::optional<std::string> validate_sampling(const HypSamplingConfig* c, uint32_t vocab) {
    if (c == nullptr || c->temperature == 0.0f) return std::nullopt;
    if (c->temperature < 0.0f) return std::string("sampling temperature must be >= 0 (0 = greedy)");
    if (c->top_k < 0) return std::string("sampling top_k must be >= 0 (0 = disabled)");
    if (c->top_k > 0 && static_cast<uint64_t>(c->top_k) > vocab) return std::string("sampling top_k exceeds the vocabulary size");
    if (!std::isnan(c->top_p) && (c->top_p < 0.0f || c->top_p > 1.0f))
        return std::string("sampling top_p must be in [0, 1] (0 = disabled)");
    if (c->min_p < 0.0f || c->min_p >= 1.0f) return std::string("sampling min_p must be in [0, 1) (0 = disabled)");
    return std::nullopt;
}

// The device sampler's settings for one step: the call's config with the step's seed.
hyb::SampleSpec sample_spec(const HypSamplingConfig& c, uint64_t seed) {
    hyb::SampleSpec sp;
    sp.temperature = c.temperature;
    sp.top_k = c.top_k;
    sp.top_p = std::isnan(c.top_p) ? 0.f : c.top_p;
    sp.min_p = c.min_p;
    sp.seed = seed;
    return sp;
}

// Predictive admission before any work (the reference's governor, model.cc:665-683,
// governor.h:148-186): the call's transient device bytes (staged global caches, ring
// backups, new workspace) must fit under the model's memory budget on top of the bytes
// already allocated, and in the device's free memory with a 1 GiB reserve. A rejected
// call does nothing: the state and its cursor are untouched.
bool admit(const hyb::Model& m, const hyb::KvState& kv, uint32_t n_tokens, std::string& why) {
    uint64_t call = 0;
    if (!m.predict_call_bytes(kv, n_tokens, &call)) {
        why = "KV operation exceeds representable cache dimensions";
        return false;
    }
    const uint64_t budget = m.memory_budget();
    const uint64_t active = hyb::dev_active_bytes();
    if (budget > 0 && active + call > budget) {
        why = "predicted peak of " + std::to_string(active + call) + " device bytes exceeds the memory budget of " +
              std::to_string(budget) + " bytes";
        return false;
    }
    if (call == 0) return true;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) {
        (void)cudaGetLastError();
        return true;
    }
    if (call + (1ull << 30) > free_b) {
        why = "predicted KV growth exceeds the device memory budget";
        return false;
    }
    return true;
}

void maybe_inject_fault() {
    if (g_fault_armed) {
        g_fault_armed = false;
        throw std::runtime_error("injected post-append forward failure");
    }
}

HypStatus load_common(HypModel model, const HypGeometryParams* geometry, const char* path, bool synthetic,
                      uint64_t seed) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    if (geometry == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "geometry is null");
    if (!synthetic && path == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "weights_path is null");
    if (model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is already loaded");
    hyb::Geometry g;
    if (auto e = hyb::geometry_from_abi(*geometry, g)) return fail(HYP_STATUS_INVALID_ARGUMENT, *e);
    if (auto e = hyb::geometry_validate(g)) return fail(HYP_STATUS_INVALID_ARGUMENT, *e);
    if (!synthetic && !std::filesystem::is_directory(path))
        return fail(HYP_STATUS_NOT_FOUND, "weights artifact directory not found");
    if (auto e = hyb::geometry_engine_support(g)) return fail(HYP_STATUS_UNSUPPORTED, *e);
    return guarded("hyp_model_load", [&]() -> HypStatus {
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
            (void)cudaGetLastError();
            return fail(HYP_STATUS_UNSUPPORTED, "no CUDA device is available");
        }
        auto m = std::make_unique<hyb::Model>();
        if (model->tp_size > 1) m->set_tensor_parallel(model->tp_rank, model->tp_size, model->tp_id);
        if (synthetic) m->load_synthetic(g, seed);
        else m->load_dir(g, path);
        model->model = std::move(m);
        model->loaded = true;
        return ok();
    });
}

// ---- canary probes
__global__ void canary_sum_kernel(const float* in, float* out) {
    float s = 0.f;
    for (int i = 0; i < 4; ++i) s += in[i];
    *out = s;
}
__global__ void canary_add_one_kernel(float* v) { *v += 1.0f; }

void copy_str(char* dst, size_t cap, const std::string& s) {
    if (cap == 0) return;
    const size_t n = std::min(cap - 1, s.size());
    std::memcpy(dst, s.data(), n);
    dst[n] = '\0';
}

}  // namespace

extern "C" {

HypStatus hyp_runtime_canary(HypCanaryInfo* out) {
    if (out == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "hyp_runtime_canary requires a non-null output pointer");
    return guarded("hyp_runtime_canary", [&]() -> HypStatus {
        *out = HypCanaryInfo{};
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
            (void)cudaGetLastError();
            return fail(HYP_STATUS_UNSUPPORTED, "no CUDA device is available");
        }
        int dev = 0;
        HYB_CUDA(cudaGetDevice(&dev));
        cudaDeviceProp prop{};
        HYB_CUDA(cudaGetDeviceProperties(&prop, dev));
        if (prop.major < 10) return fail(HYP_STATUS_UNSUPPORTED, "the engine requires an sm_100 (Blackwell) GPU");
        int rt = 0, drv = 0;
        HYB_CUDA(cudaRuntimeGetVersion(&rt));
        HYB_CUDA(cudaDriverGetVersion(&drv));
        size_t free_b = 0, total_b = 0;
        HYB_CUDA(cudaMemGetInfo(&free_b, &total_b));
        float host[4] = {1.f, 1.f, 1.f, 1.f};
        float* d = nullptr;
        HYB_CUDA(cudaMalloc(&d, 8 * sizeof(float)));
        float sum = 0.f, probe = 41.f;
        HYB_CUDA(cudaMemcpy(d, host, sizeof(host), cudaMemcpyHostToDevice));
        canary_sum_kernel<<<1, 1>>>(d, d + 4);
        HYB_CUDA(cudaMemcpy(d + 5, &probe, sizeof(float), cudaMemcpyHostToDevice));
        canary_add_one_kernel<<<1, 1>>>(d + 5);
        HYB_CUDA(cudaGetLastError());
        HYB_CUDA(cudaMemcpy(&sum, d + 4, sizeof(float), cudaMemcpyDeviceToHost));
        HYB_CUDA(cudaMemcpy(&probe, d + 5, sizeof(float), cudaMemcpyDeviceToHost));
        cudaFree(d);
        if (std::fabs(sum - 4.f) > 1e-4f) return fail(HYP_STATUS_INTERNAL, "CUDA tensor canary returned the wrong value");
        if (std::fabs(probe - 42.f) > 1e-4f) return fail(HYP_STATUS_INTERNAL, "CUDA kernel canary returned the wrong value");
        out->abi_version = kAbiVersion;
        out->mlx_compile_major = CUDART_VERSION / 1000;
        out->mlx_compile_minor = (CUDART_VERSION % 1000) / 10;
        out->mlx_compile_patch = CUDART_VERSION % 10;
        out->macos_major = static_cast<uint32_t>(drv / 1000);
        out->macos_minor = static_cast<uint32_t>((drv % 1000) / 10);
        out->macos_patch = static_cast<uint32_t>(drv % 10);
        out->gpu_family = static_cast<uint32_t>(prop.major * 10 + prop.minor);
        out->recommended_working_set_bytes = total_b;
        out->effective_budget_bytes = free_b;
        out->soft_watermark_bytes = free_b / 10 * 9;
        out->mlx_probe_value = sum;
        out->metallib_probe_value = probe;
        copy_str(out->mlx_runtime_version, sizeof(out->mlx_runtime_version),
                 "cuda " + std::to_string(rt / 1000) + "." + std::to_string((rt % 1000) / 10));
        copy_str(out->gpu_name, sizeof(out->gpu_name), prop.name);
        return ok();
    });
}

HypStatus hyp_last_error(char* buffer, size_t len) {
    if (buffer == nullptr || len == 0) return fail(HYP_STATUS_INVALID_ARGUMENT, "hyp_last_error requires a writable non-empty buffer");
    std::snprintf(buffer, len, "%s", g_last_error);
    return HYP_STATUS_OK;
}

HypStatus hyp_model_create(HypModel* out) { return create_handle(out, kModelMagic); }
HypStatus hyp_model_free(HypModel* m) { return free_handle(m, kModelMagic); }

HypStatus hyp_model_load(HypModel model, const HypGeometryParams* geometry, const char* weights_path) {
    return load_common(model, geometry, weights_path, false, 0);
}

HypStatus hyp_kvstate_create(HypModel model, HypKvState* out) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    if (out == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "out_kvstate is null");
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded; cannot allocate KV state");
    return guarded("hyp_kvstate_create", [&]() -> HypStatus {
        DeviceGuard dg(model->model->device());
        auto kv = model->model->new_kv();
        auto* h = new HypKvStateOpaque{};
        h->magic = kKvStateMagic;
        h->kv = std::move(kv);
        h->owner = model;
        *out = h;
        return ok();
    });
}

HypStatus hyp_kvstate_free(HypKvState* kv) { return free_handle(kv, kKvStateMagic); }

}  // extern "C"

namespace {

// Shared prefill driver (greedy or sampled; optional logits copy-out).
HypStatus prefill_impl(HypModel model, HypKvState kv, const HypTokenStream* tokens, const HypSamplingConfig* cfg,
                       HypStepResult out, void* host_logits) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    st = validate_kv(kv);
    if (st != HYP_STATUS_OK) return st;
    if (tokens == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "tokens is null");
    if (tokens->count == 0) return fail(HYP_STATUS_INVALID_ARGUMENT, "prefill token count is 0");
    if (tokens->tokens == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "tokens->tokens is null");
    st = validate_result(out);
    if (st != HYP_STATUS_OK) return st;
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    if (kv->kv->offset != 0) return fail(HYP_STATUS_INVALID_ARGUMENT, "prefill requires a fresh (offset 0) KV state");
    hyb::Model& m = *model->model;
    for (uint32_t i = 0; i < tokens->count; ++i)
        if (tokens->tokens[i] >= m.geometry().vocab) return fail(HYP_STATUS_INVALID_ARGUMENT, "token id is outside the vocabulary");
    return guarded("hyp_prefill_chunk", [&]() -> HypStatus {
        DeviceGuard dg(m.device());
        std::string why;
        if (!admit(m, *kv->kv, tokens->count, why)) {
            write_result(out, nullptr, 0, HYP_GOVERNOR_HARD_REJECT, m, *kv->kv, false);
            return fail(HYP_STATUS_OOM_GOVERNOR, why);
        }
        hyb::dev_reset_peak();
        const bool sampled = cfg != nullptr && cfg->temperature != 0.0f;
        std::vector<uint16_t> logits;
        hyb::StepOut o;
        // a fresh state always grows its global caches: the call is staged, and a failure
        // leaves the state fresh (model.cc:531-600)
        hyb::KvTransaction tx = m.begin_kv_transaction(*kv->kv, tokens->count);
        const hyb::SampleSpec spec = sampled ? sample_spec(*cfg, cfg->seed) : hyb::SampleSpec{};
        try {
            o = m.prefill(*kv->kv, tokens->tokens, tokens->count, host_logits ? &logits : nullptr,
                          sampled ? &spec : nullptr);
            maybe_inject_fault();
        } catch (...) {
            if (tx.active) m.rollback_kv_transaction(*kv->kv, tx);
            else kv->kv->poisoned = true;  // cache contents are partially written
            throw;
        }
        tx = hyb::KvTransaction{};  // publish (a fresh state kept no buffers worth freeing)
        if (host_logits) std::memcpy(host_logits, logits.data(), logits.size() * 2);
        write_result(out, &o, o.near_tie ? 1u : 0u, HYP_GOVERNOR_READY, m, *kv->kv, sampled);
        return ok();
    });
}

HypStatus decode_impl(HypModel model, HypKvState kv, uint32_t n_tokens, const HypSamplingConfig* cfg,
                      HypStepResult out, void* host_logits, const uint32_t* forced) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    st = validate_kv(kv);
    if (st != HYP_STATUS_OK) return st;
    st = validate_result(out);
    if (st != HYP_STATUS_OK) return st;
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    if (kv->kv->offset == 0) return fail(HYP_STATUS_INVALID_ARGUMENT, "decode requires a populated KV state (prefill first)");
    hyb::Model& m = *model->model;
    if (n_tokens == 0) {
        write_result(out, nullptr, 0, HYP_GOVERNOR_READY, m, *kv->kv, cfg != nullptr && cfg->temperature != 0.0f);
        return ok();
    }
    if (forced && *forced >= m.geometry().vocab) return fail(HYP_STATUS_INVALID_ARGUMENT, "token id is outside the vocabulary");
    return guarded("hyp_decode_block", [&]() -> HypStatus {
        DeviceGuard dg(m.device());
        std::string why;
        if (!admit(m, *kv->kv, n_tokens, why)) {
            write_result(out, nullptr, 0, HYP_GOVERNOR_HARD_REJECT, m, *kv->kv, false);
            return fail(HYP_STATUS_OOM_GOVERNOR, why);
        }
        hyb::dev_reset_peak();
        const bool sampled = cfg != nullptr && cfg->temperature != 0.0f;
        uint64_t rng = sampled ? cfg->seed : 0;
        uint32_t near_ties = 0;
        hyb::StepOut o;
        std::vector<uint16_t> logits;
        // a block that grows a global cache runs staged and rolls back on failure; one
        // that does not runs directly and a failure consumes the state (model.cc:79-105,
        // 684-735)
        hyb::KvTransaction tx = m.begin_kv_transaction(*kv->kv, n_tokens);
        for (uint32_t step = 0; step < n_tokens; ++step) {
            if (forced) kv->kv->last_token = *forced;
            const hyb::SampleSpec spec = sampled ? sample_spec(*cfg, rng) : hyb::SampleSpec{};
            try {
                o = m.decode_step(*kv->kv, host_logits ? &logits : nullptr, sampled ? &spec : nullptr);
                if (step == 0) maybe_inject_fault();
            } catch (...) {
                if (tx.active) m.rollback_kv_transaction(*kv->kv, tx);
                else kv->kv->poisoned = true;
                throw;
            }
            if (sampled) rng = rng * 6364136223846793005ULL + 1442695040888963407ULL;  // model.cc:944
            if (o.near_tie) ++near_ties;
        }
        tx = hyb::KvTransaction{};  // publish: free the live buffers the staged ones replaced
        if (host_logits) std::memcpy(host_logits, logits.data(), logits.size() * 2);
        write_result(out, &o, near_ties, HYP_GOVERNOR_READY, m, *kv->kv, sampled);
        return ok();
    });
}

}  // namespace

extern "C" {

HypStatus hyp_prefill_chunk(HypModel model, HypKvState kv, const HypTokenStream* tokens, HypStepResult out) {
    return prefill_impl(model, kv, tokens, nullptr, out, nullptr);
}

HypStatus hyp_decode_block(HypModel model, HypKvState kv, uint32_t n_tokens, HypStepResult out) {
    return decode_impl(model, kv, n_tokens, nullptr, out, nullptr, nullptr);
}

HypStatus hyp_prefill_chunk_sampled(HypModel model, HypKvState kv, const HypTokenStream* tokens,
                                    const HypSamplingConfig* config, HypStepResult out) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    st = validate_kv(kv);
    if (st != HYP_STATUS_OK) return st;
    st = validate_result(out);
    if (st != HYP_STATUS_OK) return st;
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    if (auto e = validate_sampling(config, model->model->geometry().vocab)) return fail(HYP_STATUS_INVALID_ARGUMENT, *e);
    if (config == nullptr || config->temperature == 0.0f) return hyp_prefill_chunk(model, kv, tokens, out);
    return prefill_impl(model, kv, tokens, config, out, nullptr);
}

HypStatus hyp_decode_block_sampled(HypModel model, HypKvState kv, uint32_t n_tokens, const HypSamplingConfig* config,
                                   HypStepResult out) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    st = validate_kv(kv);
    if (st != HYP_STATUS_OK) return st;
    st = validate_result(out);
    if (st != HYP_STATUS_OK) return st;
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    if (auto e = validate_sampling(config, model->model->geometry().vocab)) return fail(HYP_STATUS_INVALID_ARGUMENT, *e);
    if (config == nullptr || config->temperature == 0.0f) return hyp_decode_block(model, kv, n_tokens, out);
    return decode_impl(model, kv, n_tokens, config, out, nullptr, nullptr);
}

HypStatus hyp_step_result_create(HypStepResult* out) { return create_handle(out, kStepResultMagic); }
HypStatus hyp_step_result_free(HypStepResult* r) { return free_handle(r, kStepResultMagic); }

HypStatus hyp_step_result_fields(HypStepResult r, HypStepResultFields* out) {
    if (out == nullptr) return HYP_STATUS_INVALID_ARGUMENT;
    if (r == nullptr || r->magic != kStepResultMagic) return HYP_STATUS_INVALID_ARGUMENT;
    *out = r->fields;
    return HYP_STATUS_OK;
}

// ------------------------------------------------------------------ extensions (hyperion_b200.h)
HypStatus hyb_model_load_synthetic(HypModel model, const HypGeometryParams* geometry, uint64_t seed) {
    return load_common(model, geometry, nullptr, true, seed);
}

HypStatus hyb_model_stream(HypModel model, void** out_stream) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    if (out_stream == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "out_stream is null");
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    *out_stream = model->model->stream();
    return ok();
}

HypStatus hyb_kvstate_clone(HypModel model, HypKvState src, uint32_t last_token, HypKvState* out) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    st = validate_kv(src);
    if (st != HYP_STATUS_OK) return st;
    if (out == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "out is null");
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    if (src->owner != model) return fail(HYP_STATUS_INVALID_ARGUMENT, "kvstate belongs to another model");
    hyb::Model& m = *model->model;
    if (last_token != UINT32_MAX && last_token >= m.geometry().vocab)
        return fail(HYP_STATUS_INVALID_ARGUMENT, "token id is outside the vocabulary");
    return guarded("hyb_kvstate_clone", [&]() -> HypStatus {
        DeviceGuard dg(m.device());
        auto kv = m.clone_kv(*src->kv, last_token == UINT32_MAX ? src->kv->last_token : last_token);
        auto* h = new HypKvStateOpaque{};
        h->magic = kKvStateMagic;
        h->kv = std::move(kv);
        h->owner = model;
        *out = h;
        return ok();
    });
}

HypStatus hyb_decode_batch(HypModel model, const HypKvState* kvstates, uint32_t n, uint32_t* tokens_out,
                           float* logits_out) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    if (kvstates == nullptr || tokens_out == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "null argument");
    if (n == 0 || n > static_cast<uint32_t>(hyb::kMaxDecodeBatch))
        return fail(HYP_STATUS_INVALID_ARGUMENT, "batch must hold 1 to 64 states");
    for (uint32_t i = 0; i < n; ++i) {
        st = validate_kv(kvstates[i]);
        if (st != HYP_STATUS_OK) return st;
        if (kvstates[i]->owner != model) return fail(HYP_STATUS_INVALID_ARGUMENT, "kvstate belongs to another model");
        if (kvstates[i]->kv->offset == 0)
            return fail(HYP_STATUS_INVALID_ARGUMENT, "decode requires a populated KV state (prefill first)");
        for (uint32_t j = 0; j < i; ++j)
            if (kvstates[j] == kvstates[i]) return fail(HYP_STATUS_INVALID_ARGUMENT, "a kvstate appears twice in the batch");
    }
    hyb::Model& m = *model->model;
    return guarded("hyb_decode_batch", [&]() -> HypStatus {
        DeviceGuard dg(m.device());
        std::string why;
        for (uint32_t i = 0; i < n; ++i)
            if (!admit(m, *kvstates[i]->kv, 1, why)) return fail(HYP_STATUS_OOM_GOVERNOR, why);
        std::vector<hyb::KvState*> ks(n);
        for (uint32_t i = 0; i < n; ++i) ks[i] = kvstates[i]->kv.get();
        std::vector<hyb::StepOut> outs(n);
        try {
            m.decode_batch(ks.data(), static_cast<int>(n), outs.data());
        } catch (...) {
            for (auto* k : ks) k->poisoned = true;  // a failed step consumes every state of the batch
            throw;
        }
        for (uint32_t i = 0; i < n; ++i) {
            tokens_out[i] = outs[i].token;
            if (logits_out) logits_out[i] = outs[i].logit;
        }
        return ok();
    });
}

HypStatus hyb_verify(HypModel model, HypKvState kv, const uint32_t* draft, uint32_t n_draft, uint32_t* tokens_out,
                     float* logits_out, uint32_t* n_accepted) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    st = validate_kv(kv);
    if (st != HYP_STATUS_OK) return st;
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    if (kv->owner != model) return fail(HYP_STATUS_INVALID_ARGUMENT, "kvstate belongs to another model");
    if (draft == nullptr || tokens_out == nullptr || n_accepted == nullptr)
        return fail(HYP_STATUS_INVALID_ARGUMENT, "null argument");
    if (n_draft == 0 || n_draft > static_cast<uint32_t>(hyb::kSpecMax))
        return fail(HYP_STATUS_INVALID_ARGUMENT, "verify takes 1 to 8 draft tokens");
    if (kv->kv->offset == 0) return fail(HYP_STATUS_INVALID_ARGUMENT, "decode requires a populated KV state (prefill first)");
    hyb::Model& m = *model->model;
    for (uint32_t i = 0; i < n_draft; ++i)
        if (draft[i] >= m.geometry().vocab) return fail(HYP_STATUS_INVALID_ARGUMENT, "token id is outside the vocabulary");
    return guarded("hyb_verify", [&]() -> HypStatus {
        DeviceGuard dg(m.device());
        std::string why;
        if (!admit(m, *kv->kv, n_draft + 1, why)) return fail(HYP_STATUS_OOM_GOVERNOR, why);
        std::vector<hyb::StepOut> outs(n_draft + 1);
        int a = 0;
        try {
            a = m.verify(*kv->kv, draft, static_cast<int>(n_draft), outs.data());
        } catch (...) {
            kv->kv->poisoned = true;  // a failed step consumes the state, as a failed decode does
            throw;
        }
        for (uint32_t i = 0; i <= n_draft; ++i) {
            tokens_out[i] = outs[i].token;
            if (logits_out) logits_out[i] = outs[i].logit;
        }
        *n_accepted = static_cast<uint32_t>(a);
        return ok();
    });
}

HypStatus hyb_nccl_unique_id(void* out128) {
    if (out128 == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "output buffer is null");
    return guarded("hyb_nccl_unique_id", [&]() -> HypStatus {
        hyb::TpComm::unique_id(out128);
        return ok();
    });
}

HypStatus hyb_model_set_tensor_parallel(HypModel model, int32_t rank, int32_t size, const void* unique_id) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    if (model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "tensor parallelism must be set before hyp_model_load");
    if (size < 1 || size > 8 || rank < 0 || rank >= size)
        return fail(HYP_STATUS_INVALID_ARGUMENT, "tensor parallel rank/size out of range (size 1..8)");
    if (size > 1 && unique_id == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "unique_id is null");
    model->tp_rank = rank;
    model->tp_size = size;
    if (unique_id) std::memcpy(model->tp_id, unique_id, sizeof(model->tp_id));
    return ok();
}

HypStatus hyb_model_set_attention_rounding(HypModel model, int32_t mode) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    if (mode != 0 && mode != 1) return fail(HYP_STATUS_INVALID_ARGUMENT, "attention rounding mode must be 0 or 1");
    model->model->set_attention_rounding(mode);
    return ok();
}

HypStatus hyb_model_set_memory_budget(HypModel model, uint64_t bytes) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    model->model->set_memory_budget(bytes);
    return ok();
}

HypStatus hyb_model_weight_bytes(HypModel model, uint64_t* resident, uint64_t* algorithmic, uint64_t* scratch) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    if (!model->loaded) return fail(HYP_STATUS_INVALID_ARGUMENT, "model is not loaded");
    if (resident) *resident = model->model->weight_bytes_resident();
    if (algorithmic) *algorithmic = model->model->weight_bytes_algorithmic();
    if (scratch) *scratch = model->model->unpack_scratch_bytes();
    return ok();
}

HypStatus hyb_kv_cursor(HypKvState kv, uint32_t* offset, uint32_t* last_token) {
    if (kv == nullptr || kv->magic != kKvStateMagic) return fail(HYP_STATUS_INVALID_ARGUMENT, "kvstate handle is invalid");
    if (offset) *offset = kv->kv->offset;
    if (last_token) *last_token = kv->kv->last_token;
    return ok();
}

HypStatus hyb_kv_copy_layer(HypModel model, HypKvState kv, uint32_t layer, int32_t which, void* host_out, uint32_t* rows) {
    HypStatus st = validate_model(model);
    if (st != HYP_STATUS_OK) return st;
    if (kv == nullptr || kv->magic != kKvStateMagic) return fail(HYP_STATUS_INVALID_ARGUMENT, "kvstate handle is invalid");
    if (!model->loaded || rows == nullptr) return fail(HYP_STATUS_INVALID_ARGUMENT, "model not loaded or rows is null");
    const hyb::Geometry& g = model->model->geometry();
    if (layer >= g.n_layers) return fail(HYP_STATUS_INVALID_ARGUMENT, "layer out of range");
    return guarded("hyb_kv_copy_layer", [&]() -> HypStatus {
        DeviceGuard dg(model->model->device());
        size_t li = 0, gi = 0;
        for (uint32_t i = 0; i < layer; ++i) (g.kinds[i] == hyb::LayerKind::Sliding ? li : gi)++;
        const hyb::bf16* src;
        uint32_t cap;
        size_t row;
        if (g.kinds[layer] == hyb::LayerKind::Sliding) {
            const auto& c = kv->kv->local[li];
            src = which == 0 ? c.k : c.v;
            cap = c.cap;
            row = static_cast<size_t>(c.nkv) * c.hd;
        } else {
            const auto& c = kv->kv->global[gi];
            src = which == 0 ? c.k : c.v;
            cap = c.capacity;
            row = static_cast<size_t>(c.nkv) * c.hd;
        }
        const uint32_t n = std::min(cap, *rows);
        if (host_out && n > 0) HYB_CUDA(cudaMemcpy(host_out, src, n * row * 2, cudaMemcpyDeviceToHost));
        *rows = cap;
        return ok();
    });
}

HypStatus hyb_prefill_logits(HypModel model, HypKvState kv, const HypTokenStream* tokens, HypStepResult out,
                             void* host_logits) {
    return prefill_impl(model, kv, tokens, nullptr, out, host_logits);
}

HypStatus hyb_decode_logits(HypModel model, HypKvState kv, HypStepResult out, void* host_logits) {
    return decode_impl(model, kv, 1, nullptr, out, host_logits, nullptr);
}

HypStatus hyb_decode_forced(HypModel model, HypKvState kv, uint32_t token, HypStepResult out, void* host_logits) {
    return decode_impl(model, kv, 1, nullptr, out, host_logits, &token);
}

// Test hook: the next decode throws once after its first forward (host-side fault,
// no device involvement), like the reference's post-append fault (test_fault.cc).
HypStatus hyb_test_arm_post_append_fault(void) {
    g_fault_armed = true;
    return ok();
}

}  // extern "C"
