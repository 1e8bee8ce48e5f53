"""Op-level calls into libhyperion_mlx.so on torch CUDA tensors.

torch is used only to own device memory and streams; every computation runs in
the library's sm_100a kernels through the hyperion_b200.h C ABI.
"""
from __future__ import annotations

import ctypes

import torch

from . import check, lib


def _p(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream=None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """y = x @ dequant(w).T for affine Q4/g64 (x bf16 [M,K], w int32/uint32 [N,K/8])."""
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    check(lib().hyb_quantized_matmul(_p(x), _p(w), _p(scales), _p(biases), _p(out), M, K, N, 64, 4,
                                     _stream(stream)))
    return out


def qmv_fused(x, w, scales, biases, prologue=0, epilogue=0, norm_w=None, resid=None, post_w=None, scalar=None,
              h_out=None, eps=1e-6, out=None, stream=None):
    """Batch-1 qmv with the decode engine's fused norm prologue / GeGLU epilogue."""
    K = x.numel()
    N = w.shape[0]
    if out is None:
        out = torch.empty(N // 2 if epilogue == 1 else N, dtype=torch.bfloat16, device=x.device)
    opt = lambda t: _p(t) if t is not None else None
    check(lib().hyb_qmv_fused(_p(x), _p(w), _p(scales), _p(biases), _p(out), K, N, prologue, epilogue,
                              opt(norm_w), opt(resid), opt(post_w), opt(scalar), opt(h_out), eps, _stream(stream)))
    return out


def qmv_pack(w, scales, biases, stream=None) -> torch.Tensor:
    """Repack MLX-layout Q4/g64 weights into the decode engine's packed layout (uint8 tensor)."""
    N, K8 = w.shape
    K = K8 * 8
    out = torch.empty(lib().hyb_qmv_packed_bytes(K, N), dtype=torch.uint8, device=w.device)
    check(lib().hyb_qmv_pack(_p(w), _p(scales), _p(biases), K, N, _p(out), _stream(stream)))
    return out


def qmv_unpack(packed, K, N, stream=None):
    """The MLX layout (w [N, K/8] uint32, scales/biases [N, K/64] bf16) of a packed matrix."""
    w = torch.empty((N, K // 8), dtype=torch.int32, device=packed.device)
    s = torch.empty((N, K // 64), dtype=torch.bfloat16, device=packed.device)
    b = torch.empty((N, K // 64), dtype=torch.bfloat16, device=packed.device)
    check(lib().hyb_qmv_unpack(_p(packed), K, N, _p(w), _p(s), _p(b), _stream(stream)))
    return w, s, b


def embed_packed(ids, packed, H, N, embed_scale_bits, stream=None):
    """Embedding rows of a packed [N, H] table (dequantised, x embed scale): [L, H] bf16."""
    L = ids.numel()
    out = torch.empty((L, H), dtype=torch.bfloat16, device=packed.device)
    check(lib().hyb_embed_packed(_p(ids), L, _p(packed), H, N, embed_scale_bits, _p(out), _stream(stream)))
    return out


def qmv_packed(x, packed, K, N, prologue=0, epilogue=0, norm_w=None, resid=None, post_w=None, scalar=None,
               h_out=None, eps=1e-6, out=None, stream=None):
    """Batch-1 qmv over packed weights (TMA-streamed kernel), same options as qmv_fused."""
    if out is None:
        out = torch.empty(N // 2 if epilogue == 1 else N, dtype=torch.bfloat16, device=x.device)
    opt = lambda t: _p(t) if t is not None else None
    check(lib().hyb_qmv_packed(_p(x), _p(packed), _p(out), K, N, prologue, epilogue, opt(norm_w), opt(resid),
                               opt(post_w), opt(scalar), opt(h_out), eps, _stream(stream)))
    return out


def qmv_batched(x, packed, K, N, geglu=False, out=None, stream=None):
    """Batched decode qmv over packed weights: x [B, K] bf16 -> [B, N] (or [B, N/2] with GeGLU)."""
    B = x.shape[0]
    if out is None:
        out = torch.empty((B, N // 2 if geglu else N), dtype=torch.bfloat16, device=x.device)
    check(lib().hyb_qmv_batched(_p(x), B, x.stride(0), _p(packed), _p(out), out.stride(0), K, N, 1 if geglu else 0,
                                _stream(stream)))
    return out


class DecodeScratch:
    """Device workspace for hyb_sdpa_decode (zeroed once)."""

    def __init__(self, n_heads, n_kv, hd, max_keys, device="cuda"):
        n = lib().hyb_sdpa_decode_scratch_bytes(n_heads, n_kv, hd, max_keys)
        self.buf = torch.zeros(n, dtype=torch.uint8, device=device)
        self.nbytes = n


def sdpa_decode(q, k_cache, v_cache, last_pos: int, n_keys: int, scratch: DecodeScratch, scale=1.0,
                softcap=0.0, rounding=0, out=None, stream=None):
    H, hd = q.shape
    cap, nkv, _ = k_cache.shape
    if out is None:
        out = torch.empty_like(q)
    check(lib().hyb_sdpa_decode(_p(q), _p(k_cache), _p(v_cache), _p(out), H, nkv, hd, cap, last_pos, n_keys,
                                scale, softcap, rounding, _p(scratch.buf), scratch.nbytes, _stream(stream)))
    return out


def sdpa_decode_fused(qkv, v_from_k, q_norm, k_norm, inv_freq, k_cache, v_cache, pos, n_keys, n_heads, eps=1e-6,
                      scale=1.0, softcap=0.0, rounding=0, out=None, stream=None):
    """Fused decode step: norms + RoPE + cache append + attention (cluster kernel)."""
    cap, nkv, hd = k_cache.shape
    if out is None:
        out = torch.empty((n_heads, hd), dtype=torch.bfloat16, device=qkv.device)
    check(lib().hyb_sdpa_decode_fused(_p(qkv), int(v_from_k), _p(q_norm), _p(k_norm), _p(inv_freq), eps,
                                      _p(k_cache), _p(v_cache), cap, pos, n_keys, n_heads, nkv, hd, scale, softcap,
                                      rounding, _p(out), _stream(stream)))
    return out


def sdpa_prefill(q, k, v, q_pos0: int, k_pos0: int, window: int, scale=1.0, softcap=0.0, rounding=0,
                 out=None, stream=None):
    Lq, H, hd = q.shape
    Lk, nkv, _ = k.shape
    if out is None:
        out = torch.empty_like(q)
    check(lib().hyb_sdpa_prefill(_p(q), _p(k), _p(v), _p(out), Lq, Lk, H, nkv, hd, q_pos0, k_pos0, window,
                                 scale, softcap, rounding, _stream(stream)))
    return out


def rms_norm(x, w, eps=1e-6, out=None, stream=None):
    rows = x.numel() // x.shape[-1]
    if out is None:
        out = torch.empty_like(x)
    check(lib().hyb_rms_norm(_p(x), _p(w) if w is not None else None, _p(out), rows, x.shape[-1], eps,
                             _stream(stream)))
    return out


def qkv_post(qkv, n_heads, n_kv, hd, v_from_k, q_norm, k_norm, inv_freq, pos0, eps=1e-6, k_cache=None,
             v_cache=None, cache_first=0, stream=None):
    L, ld = qkv.shape
    q_out = torch.empty((L, n_heads, hd), dtype=torch.bfloat16, device=qkv.device)
    k_out = torch.empty((L, n_kv, hd), dtype=torch.bfloat16, device=qkv.device)
    v_out = torch.empty((L, n_kv, hd), dtype=torch.bfloat16, device=qkv.device)
    cap = k_cache.shape[0] if k_cache is not None else 0
    check(lib().hyb_qkv_post(_p(qkv), L, ld, n_heads, n_kv, hd, int(v_from_k), _p(q_norm), _p(k_norm),
                             _p(inv_freq), pos0, eps, _p(q_out), _p(k_out), _p(v_out),
                             _p(k_cache) if k_cache is not None else None,
                             _p(v_cache) if v_cache is not None else None, cap, cache_first, _stream(stream)))
    return q_out, k_out, v_out
