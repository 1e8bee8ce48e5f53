"""Seeded synthetic Gemma-style checkpoints and geometries (the BASELINE configs).

Weights follow the distributions the benchmark configurations specify:
  * every projection is MLX affine Q4/g64: codes q ~ U{0..15} packed 8 per
    uint32 along K (code i of word j in bits [4i, 4i+4)), scales
    s = bf16(|N(0, 0.02)|), biases b = -8 * s;
  * the tied embedding table is a bf16 N(0, 0.02) matrix quantized with the
    affine g64/b4 rule (per group: range / 15 scale anchored at the
    larger-magnitude edge, as MLX's ``quantize`` does);
  * RMSNorm weights are stored as bf16(1 + N(0, 0.02)) - the "(1 + w)" Gemma
    scaling folded into the tensor, so the engine multiplies by the stored
    weight exactly as the reference does (forward.cc:25-27);
  * layer_scalar = bf16(1 + N(0, 0.02)).
Global (full-attention) layers omit ``v_proj``: the reference derives the layer
kind from v_proj presence (weights_loader.cc:117-127) and uses V = v_norm(k_proj).
Tensor names are the mlx-lm converted names the reference loader requires
(weights_loader.cc:141-145, 257-277).
"""
from __future__ import annotations

import dataclasses
import os
from typing import Dict, List, Optional

import numpy as np

from .safetensors_io import write_safetensors

try:
    import ml_dtypes

    _BF16 = ml_dtypes.bfloat16
except ImportError:  # pragma: no cover
    _BF16 = None


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclasses.dataclass
class Geometry:
    """The subset of HypGeometryParams the engine uses, with config names."""

    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    layer_types: List[int]  # 0 = sliding, 1 = full
    num_attention_heads: int
    head_dim_local: int
    head_dim_global: int
    num_kv_heads_local: int
    num_kv_heads_global: int
    sliding_window: int
    vocab_size: int
    attention_k_eq_v_global: int = 1
    rope_theta_local: float = 10000.0
    rope_theta_global: float = 1000000.0
    partial_rotary_factor_global: float = 0.25
    final_logit_softcapping: float = 30.0
    rms_norm_eps: float = 1e-6
    max_position_embeddings: int = 131072
    model_type: int = 1

    def head_dim(self, layer: int) -> int:
        return self.head_dim_global if self.layer_types[layer] == 1 else self.head_dim_local

    def n_kv(self, layer: int) -> int:
        return self.num_kv_heads_global if self.layer_types[layer] == 1 else self.num_kv_heads_local


def pattern_5to1(n_layers: int) -> List[int]:
    """Global at (i+1) % 6 == 0, and the last layer forced global (geometry.cc:86-88)."""
    t = [1 if (i + 1) % 6 == 0 else 0 for i in range(n_layers)]
    t[-1] = 1
    return t


def config0() -> Geometry:
    """tiny Gemma-style decoder (2 layers, hidden 256)."""
    return Geometry(hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
                    layer_types=[0, 1], num_attention_heads=4, head_dim_local=64,
                    head_dim_global=64, num_kv_heads_local=2, num_kv_heads_global=2,
                    sliding_window=128, vocab_size=1024, max_position_embeddings=4096)


def config3(n_layers: int = 48) -> Geometry:
    """Gemma-12B-shaped decoder (hd 256 / 8 KV heads on all layers)."""
    return Geometry(hidden_size=3840, intermediate_size=15360, num_hidden_layers=n_layers,
                    layer_types=pattern_5to1(n_layers), num_attention_heads=16,
                    head_dim_local=256, head_dim_global=256, num_kv_heads_local=8,
                    num_kv_heads_global=8, sliding_window=1024, vocab_size=262144,
                    max_position_embeddings=131072)


def config4(n_layers: int = 62) -> Geometry:
    """Gemma-27B-shaped decoder (hd 128, 32 q / 16 KV heads)."""
    return Geometry(hidden_size=5376, intermediate_size=21504, num_hidden_layers=n_layers,
                    layer_types=pattern_5to1(n_layers), num_attention_heads=32,
                    head_dim_local=128, head_dim_global=128, num_kv_heads_local=16,
                    num_kv_heads_global=16, sliding_window=1024, vocab_size=262144,
                    max_position_embeddings=131072)


def tiny_fixture_geometry() -> Geometry:
    """The reference's committed gemma4-unified-tiny fixture geometry (6 layers, hidden 128)."""
    return Geometry(hidden_size=128, intermediate_size=256, num_hidden_layers=6,
                    layer_types=[0, 0, 0, 0, 0, 1], num_attention_heads=4,
                    head_dim_local=64, head_dim_global=128, num_kv_heads_local=2,
                    num_kv_heads_global=1, sliding_window=8, vocab_size=128,
                    max_position_embeddings=256)


def random_q4(rng: np.random.Generator, n: int, k: int):
    """Codes U{0..15}, s = bf16(|N(0,0.02)|), b = -8 s. Returns (w u32 [n,k/8], s, b bf16 bits)."""
    assert k % 64 == 0
    q = rng.integers(0, 16, size=(n, k), dtype=np.uint32)
    w = pack_q4(q)
    s = f32_to_bf16_bits(np.abs(rng.standard_normal((n, k // 64), dtype=np.float32) * 0.02))
    b = f32_to_bf16_bits(-8.0 * bf16_bits_to_f32(s))
    return w, s, b


def pack_q4(q: np.ndarray) -> np.ndarray:
    """Pack codes [n, k] (0..15) into u32 [n, k/8]; code 8j+i -> bits [4i, 4i+4) of word j."""
    n, k = q.shape
    q = q.astype(np.uint32).reshape(n, k // 8, 8)
    w = np.zeros((n, k // 8), dtype=np.uint32)
    for i in range(8):
        w |= q[:, :, i] << np.uint32(4 * i)
    return w


def affine_quantize(wf: np.ndarray):
    """Affine g64/b4 quantization of a float matrix [n, k] (MLX ``quantize`` rule)."""
    n, k = wf.shape
    g = wf.reshape(n, k // 64, 64).astype(np.float32)
    wmax = g.max(axis=-1, keepdims=True)
    wmin = g.min(axis=-1, keepdims=True)
    mask = np.abs(wmin) > np.abs(wmax)
    scales = np.maximum((wmax - wmin) / 15.0, 1e-7).astype(np.float32)
    scales = np.where(mask, scales, -scales)
    edge = np.where(mask, wmin, wmax)
    q0 = np.round(edge / scales)
    scales = np.where(q0 != 0, edge / np.where(q0 != 0, q0, 1), scales)
    biases = np.where(q0 == 0, 0.0, edge).astype(np.float32)
    sb = f32_to_bf16_bits(scales.reshape(n, k // 64))
    bb = f32_to_bf16_bits(biases.reshape(n, k // 64))
    q = np.clip(np.round((g - biases) / scales), 0, 15).astype(np.uint32).reshape(n, k)
    return pack_q4(q), sb, bb


def normal_bf16(rng: np.random.Generator, shape, std=0.02, mean=0.0) -> np.ndarray:
    return f32_to_bf16_bits(mean + std * rng.standard_normal(shape, dtype=np.float32))


def make_weights(geo: Geometry, seed: int = 0) -> Dict[str, np.ndarray]:
    """All tensors of a synthetic checkpoint, keyed by the mlx-lm converted names."""
    rng = np.random.default_rng(seed)
    H = geo.hidden_size
    t: Dict[str, np.ndarray] = {}

    def proj(base: str, n: int, k: int):
        w, s, b = random_q4(rng, n, k)
        t[base + ".weight"], t[base + ".scales"], t[base + ".biases"] = w, s, b

    emb = rng.standard_normal((geo.vocab_size, H), dtype=np.float32) * 0.02
    emb = bf16_bits_to_f32(f32_to_bf16_bits(emb))
    w, s, b = affine_quantize(emb)
    pre = "language_model.model."
    t[pre + "embed_tokens.weight"], t[pre + "embed_tokens.scales"], t[pre + "embed_tokens.biases"] = w, s, b
    t[pre + "norm.weight"] = normal_bf16(rng, (H,), mean=1.0)
    for i in range(geo.num_hidden_layers):
        hd, nkv = geo.head_dim(i), geo.n_kv(i)
        nh = geo.num_attention_heads
        p = f"{pre}layers.{i}."
        a = p + "self_attn."
        proj(a + "q_proj", nh * hd, H)
        proj(a + "k_proj", nkv * hd, H)
        if geo.layer_types[i] == 0:
            proj(a + "v_proj", nkv * hd, H)
        proj(a + "o_proj", H, nh * hd)
        t[a + "q_norm.weight"] = normal_bf16(rng, (hd,), mean=1.0)
        t[a + "k_norm.weight"] = normal_bf16(rng, (hd,), mean=1.0)
        for nm in ("input_layernorm", "post_attention_layernorm",
                   "pre_feedforward_layernorm", "post_feedforward_layernorm"):
            t[p + nm + ".weight"] = normal_bf16(rng, (H,), mean=1.0)
        proj(p + "mlp.gate_proj", geo.intermediate_size, H)
        proj(p + "mlp.up_proj", geo.intermediate_size, H)
        proj(p + "mlp.down_proj", H, geo.intermediate_size)
        t[p + "layer_scalar"] = normal_bf16(rng, (1,), mean=1.0)
    return t


def write_checkpoint(geo: Geometry, path: str, seed: int = 0, shards: int = 2) -> Dict[str, np.ndarray]:
    """Write a synthetic checkpoint directory (several shards, like mlx-lm output)."""
    os.makedirs(path, exist_ok=True)
    t = make_weights(geo, seed)
    names = sorted(t)
    per = (len(names) + shards - 1) // shards
    for si in range(shards):
        part = {n: t[n] for n in names[si * per:(si + 1) * per]}
        if part:
            write_safetensors(os.path.join(path, f"model-{si + 1:05d}-of-{shards:05d}.safetensors"), part)
    return t
