#include "geometry.h"

#include <cmath>

namespace hyb {

std::optional<std::string> geometry_from_abi(const HypGeometryParams& p, Geometry& g) {
    if (p.layer_types == nullptr && p.num_hidden_layers > 0) return std::string("layer_types pointer is null");
    if (p.model_type != HYP_GEMMA4_TEXT && p.model_type != HYP_GEMMA4_UNIFIED_TEXT)
        return std::string("unknown HypTextModelType");
    g.model_type = static_cast<int>(p.model_type);
    g.hidden = p.hidden_size;
    g.intermediate = p.intermediate_size;
    g.n_layers = p.num_hidden_layers;
    g.kinds.clear();
    for (uint32_t i = 0; i < p.num_hidden_layers; ++i) {
        if (p.layer_types[i] == HYP_LAYER_SLIDING) g.kinds.push_back(LayerKind::Sliding);
        else if (p.layer_types[i] == HYP_LAYER_FULL) g.kinds.push_back(LayerKind::Full);
        else return "unknown HypLayerType at index " + std::to_string(i);
    }
    g.n_heads = p.num_attention_heads;
    g.hd_local = p.head_dim_local;
    g.hd_global = p.head_dim_global;
    g.nkv_local = p.num_kv_heads_local;
    g.nkv_global = p.num_kv_heads_global;
    g.k_eq_v_global = p.attention_k_eq_v_global != 0;
    g.n_kv_shared = p.num_kv_shared_layers;
    g.window = p.sliding_window;
    auto rope = [](const HypRopeSpec& s) {
        RopeCfg r;
        r.theta = s.theta;
        r.has_partial = s.has_partial_rotary_factor != 0;
        r.partial = s.partial_rotary_factor;
        r.proportional = s.proportional != 0;
        return r;
    };
    g.rope_local = rope(p.rope_local);
    g.rope_global = rope(p.rope_global);
    g.softcap = p.final_logit_softcapping;
    g.eps = p.rms_norm_eps;
    g.attention_bias = p.attention_bias != 0;
    g.vocab = p.vocab_size;
    g.max_pos = p.max_position_embeddings;
    g.tied = p.tie_word_embeddings != 0;
    g.ple_hidden = p.ple_hidden_per_layer_input;
    g.ple_vocab = p.ple_vocab_per_layer_input;
    g.double_wide_mlp = p.use_double_wide_mlp != 0;
    g.has_moe = p.has_moe != 0;
    g.moe = p.moe;
    return std::nullopt;
}

std::optional<std::string> geometry_validate(const Geometry& g) {
    if (g.kinds.empty()) return std::string("layer_types is empty");
    if (g.kinds.size() != g.n_layers) return std::string("layer_types length does not match num_hidden_layers");
    if (g.kinds.back() != LayerKind::Full) return std::string("the last layer must be full_attention (Gemma 4 invariant)");
    if (g.n_layers == 0) return std::string("num_hidden_layers must be non-zero");
    if (g.window == 0) return std::string("sliding_window must be non-zero");
    if (g.n_kv_shared > g.n_layers) return std::string("num_kv_shared_layers exceeds num_hidden_layers");
    if (g.hd_local == 0 || g.hd_global == 0) return std::string("head_dim_local and head_dim_global must be non-zero");
    if (g.n_heads == 0 || g.nkv_local == 0 || g.nkv_global == 0)
        return std::string("attention/KV head counts must be non-zero");
    if (g.vocab == 0) return std::string("vocab_size must be non-zero");
    if (g.rope_local.proportional) return std::string("sliding rope must be the default (full rotary) scheme");
    if (g.rope_local.has_partial) return std::string("sliding rope must be full rotary (no partial_rotary_factor)");
    if (!g.rope_global.proportional) return std::string("global rope must be the proportional scheme");
    if (!g.rope_global.has_partial) return std::string("global rope must set partial_rotary_factor");
    if (g.rope_local.theta <= 0.0 || g.rope_global.theta <= 0.0) return std::string("rope_theta must be positive");
    if (!g.tied) return std::string("tie_word_embeddings must be true (lm_head is tied to the embedding table)");
    if (g.has_moe && (g.moe.num_experts == 0 || g.moe.top_k == 0 || g.moe.moe_intermediate_size == 0))
        return std::string("moe block requires non-zero num_experts/top_k/moe_intermediate_size");
    return std::nullopt;
}

std::optional<std::string> geometry_engine_support(const Geometry& g) {
    if (g.has_moe) return std::string("mixture-of-experts geometries are not supported by the CUDA engine");
    if (g.hidden % 64 != 0 || g.intermediate % 64 != 0)
        return std::string("hidden_size and intermediate_size must be multiples of 64 (Q4/g64)");
    if (g.intermediate % 16 != 0) return std::string("intermediate_size must be a multiple of 16");
    for (uint32_t hd : {g.hd_local, g.hd_global}) {
        if (hd != 64 && hd != 128 && hd != 256)
            return "head_dim " + std::to_string(hd) + " is not supported (64, 128 or 256)";
    }
    if (g.n_heads % g.nkv_local != 0 || g.n_heads % g.nkv_global != 0)
        return std::string("attention heads must be a multiple of the KV heads");
    if (g.n_heads / g.nkv_local > 8 || g.n_heads / g.nkv_global > 8)
        return std::string("GQA groups larger than 8 are not supported");
    if ((g.n_heads / g.nkv_local) * g.hd_local > 1024 || (g.n_heads / g.nkv_global) * g.hd_global > 1024)
        return std::string("GQA group x head_dim above 1024 is not supported");
    if ((g.n_heads * g.hd_local) % 64 != 0 || (g.n_heads * g.hd_global) % 64 != 0)
        return std::string("num_attention_heads * head_dim must be a multiple of 64");
    if (g.hidden * 4 > 48 * 1024) return std::string("hidden_size above 12288 is not supported");
    return std::nullopt;
}

uint32_t Geometry::rotated_dims(LayerKind k) const {
    const RopeCfg& r = k == LayerKind::Full ? rope_global : rope_local;
    const uint32_t hd = k == LayerKind::Full ? hd_global : hd_local;
    if (!r.proportional) return hd;
    uint32_t rot = static_cast<uint32_t>(r.partial * static_cast<float>(hd));
    return rot - rot % 2;
}

std::vector<float> rope_inv_freq(uint32_t hd, const RopeCfg& cfg) {
    std::vector<float> inv(hd / 2, 0.f);
    if (!cfg.proportional) {
        for (uint32_t i = 0; i < hd / 2; ++i)
            inv[i] = static_cast<float>(std::pow(cfg.theta, -2.0 * i / static_cast<double>(hd)));
    } else {
        uint32_t rot = static_cast<uint32_t>(cfg.partial * static_cast<float>(hd));
        rot -= rot % 2;
        for (uint32_t i = 0; i < rot / 2; ++i) {
            const float f = static_cast<float>(std::pow(cfg.theta, 2.0 * i / static_cast<double>(hd)));
            inv[i] = static_cast<float>(1.0 / static_cast<double>(f));
        }
    }
    return inv;
}

}  // namespace hyb
