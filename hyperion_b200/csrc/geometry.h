// Engine geometry: the validated form of HypGeometryParams plus the per-layer
// dispatch the forward pass needs.
#pragma once

#include "hyperion_mlx.h"

#include <cstdint>
#include <optional>
#include <string>
#include <vector>

namespace hyb {

enum class LayerKind : uint8_t { Sliding = 0, Full = 1 };

struct RopeCfg {
    double theta = 0;
    bool has_partial = false;
    float partial = 0.f;
    bool proportional = false;
};

struct Geometry {
    int model_type = 0;
    uint32_t hidden = 0, intermediate = 0, n_layers = 0;
    std::vector<LayerKind> kinds;
    uint32_t n_heads = 0, hd_local = 0, hd_global = 0, nkv_local = 0, nkv_global = 0;
    bool k_eq_v_global = false;
    uint32_t n_kv_shared = 0, window = 0;
    RopeCfg rope_local, rope_global;
    float softcap = 0.f, eps = 0.f;
    bool attention_bias = false;
    uint32_t vocab = 0, max_pos = 0;
    bool tied = false;
    uint32_t ple_hidden = 0, ple_vocab = 0;
    bool double_wide_mlp = false;
    bool has_moe = false;
    HypMoeConfig moe{};

    uint32_t head_dim(size_t layer) const { return kinds[layer] == LayerKind::Full ? hd_global : hd_local; }
    uint32_t n_kv(size_t layer) const { return kinds[layer] == LayerKind::Full ? nkv_global : nkv_local; }
    // Number of pairs rotated by RoPE for a layer kind (rope.cc:85-109 semantics).
    uint32_t rotated_dims(LayerKind k) const;
};

// Convert the ABI struct (reference geometry.cc:130-182 semantics). Returns an
// error message on a malformed struct.
std::optional<std::string> geometry_from_abi(const HypGeometryParams& p, Geometry& out);
// Re-check the invariants the graph needs (reference geometry.cc:185-240).
std::optional<std::string> geometry_validate(const Geometry& g);
// Extra constraints of the CUDA kernels (UNSUPPORTED when violated).
std::optional<std::string> geometry_engine_support(const Geometry& g);

// Per-pair inverse RoPE frequencies (float, hd/2 entries, 0 = identity pair).
std::vector<float> rope_inv_freq(uint32_t head_dim, const RopeCfg& cfg);

}  // namespace hyb
