"""CPU oracle for the Hyperion Gemma decode/prefill path.

TEST INFRASTRUCTURE ONLY: the parity checker and the timed host-CPU baseline.
The product path (``hyperion_b200``) never imports this module; only tests/,
``__graft_entry__.smoke()`` and bench.py's CPU legs do.

It restates, op for op and at the same bf16 rounding points, the reference
engine's forward pass (paths inside jscott3201/hyperion):
  * embed: gather + affine dequant of the tied table, times bf16(sqrt(hidden))
    (forward.cc:126-131, weights_loader.cc:181-198);
  * rms_norm: fp32 statistics, bf16(x * rsqrt(mean(x^2) + eps)) then times the
    weight in bf16; v_norm has no weight (forward.cc:25-27, 408-412);
  * RoPE: non-traditional (pairs i, i + hd/2), angle = (offset + row) * inv_freq
    in fp32; local layers rotate every pair with theta_local, global layers the
    first floor(0.25 hd)/2 pairs with the proportional exponents 2i/hd
    (rope.cc:65-123);
  * KV caches: the local ring of capacity window + 8 with slot = pos % cap and
    the logical-order window read, the global cache grown in 256-token steps
    (kv_cache.cc:161-347, kv.cc:7-96);
  * attention: masks by absolute position and the kv_len rules of
    attention_kv_len (forward.cc:46-59, 345-374, 376-508), SDPA via orc_sdpa;
  * GeGLU with every elementwise op rounded to bf16 and its constants taken as
    bf16 (forward.cc:324-343);
  * the 4-norm sandwich, residual adds and layer_scalar (forward.cc:510-542);
  * final norm, tied lm_head, bf16 softcap and the greedy scan with the
    top1 - top2 < 0.5 near-tie flag (forward.cc:133-189, model.cc:215-228);
  * chunked prefill of 2048 tokens (model.cc:574-610) and the decode loop
    (model.cc:703-718).
Quantized matmuls and attention run in the C library ``hyp_oracle.c``.
"""
from __future__ import annotations

import ctypes
import math
import os
from typing import Dict, List, Optional, Tuple

import numpy as np

from hyperion_b200.synth import Geometry, bf16_bits_to_f32, f32_to_bf16_bits

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

PREFILL_CHUNK = 2048
GAMMA_MAX = 8
GLOBAL_STEP = 256


def lib() -> ctypes.CDLL:
    """Load (building if needed) the oracle's C library."""
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            from oracle.build_oracle import build
            build()
        L = ctypes.CDLL(path)
        P = ctypes.c_void_p
        i64 = ctypes.c_int64
        L.orc_qmm.argtypes = [P, i64, i64, P, P, P, i64, P, P, ctypes.c_int]
        L.orc_qmv_fast.argtypes = [P, i64, P, P, P, i64, P, ctypes.c_int]
        L.orc_sdpa.argtypes = [P, P, P, i64, i64, i64, i64, i64, i64, i64, i64,
                               ctypes.c_float, ctypes.c_float, ctypes.c_int, P, ctypes.c_int]
        L.orc_unpack_row.argtypes = [P, i64, i64, P]
        L.orc_max_threads.restype = ctypes.c_int
        u64 = ctypes.c_uint64
        L.orc_normal_quantile.argtypes = [ctypes.c_double]
        L.orc_normal_quantile.restype = ctypes.c_double
        L.orc_normal_table.argtypes = [P]
        L.orc_synth_words.argtypes = [u64, i64, i64, i64, i64, i64, P, ctypes.c_int]
        L.orc_synth_sb.argtypes = [u64, i64, i64, i64, i64, i64, ctypes.c_float, P, P, P, ctypes.c_int]
        L.orc_synth_normal.argtypes = [u64, i64, ctypes.c_float, ctypes.c_float, P, P]
        _LIB = L
    return _LIB


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def bf(a) -> np.ndarray:
    """Round float values to bf16 bits."""
    return f32_to_bf16_bits(np.asarray(a, dtype=np.float32))


def fl(b: np.ndarray) -> np.ndarray:
    """bf16 bits -> float32."""
    return bf16_bits_to_f32(b)


# ----------------------------------------------------------------------------- ops

def qmm(x: np.ndarray, w: np.ndarray, s: np.ndarray, b: np.ndarray, nthreads: int = 0,
        want_f32: bool = False):
    """Affine Q4/g64 matmul: x bf16 [M, K] -> y bf16 [M, N] (exact-sum semantics)."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    M, K = x.shape
    N = w.shape[0]
    assert w.shape == (N, K // 8) and s.shape == (N, K // 64) and b.shape == (N, K // 64)
    w = np.ascontiguousarray(w, dtype=np.uint32)
    s = np.ascontiguousarray(s, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    y = np.empty((M, N), dtype=np.uint16)
    yf = np.empty((M, N), dtype=np.float32) if want_f32 else None
    lib().orc_qmm(_p(x), M, K, _p(w), _p(s), _p(b), N, _p(y),
                  _p(yf) if want_f32 else None, nthreads)
    return (y, yf) if want_f32 else y


def qmv_fast(x: np.ndarray, w, s, b, nthreads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16).reshape(-1)
    K = x.shape[0]
    N = w.shape[0]
    y = np.empty((N,), dtype=np.uint16)
    lib().orc_qmv_fast(_p(x), K, _p(w), _p(s), _p(b), N, _p(y), nthreads)
    return y


def sdpa(q, k, v, q_pos0: int, k_pos0: int, window: int, scale: float = 1.0,
         softcap: float = 0.0, mode: int = 0, nthreads: int = 0) -> np.ndarray:
    """q bf16 [Lq, H, D]; k, v bf16 [Lk, Hkv, D] -> bf16 [Lq, H, D]."""
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    Lq, H, D = q.shape
    Lk, Hkv, _ = k.shape
    out = np.empty_like(q)
    lib().orc_sdpa(_p(q), _p(k), _p(v), Lq, Lk, H, Hkv, D, q_pos0, k_pos0, window,
                   scale, softcap, mode, _p(out), nthreads)
    return out


def rms_norm(x: np.ndarray, w: Optional[np.ndarray], eps: float) -> np.ndarray:
    """bf16 in/out over the last axis; fp32-or-better statistics."""
    xf = fl(x).astype(np.float64)
    inv = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + np.float64(np.float32(eps)))
    t = bf((xf * inv).astype(np.float32))
    if w is None:
        return t
    return bf(fl(t) * fl(w))


def rope_inv_freq(head_dim: int, theta: float, proportional: bool, partial: float) -> np.ndarray:
    """Per-pair inverse frequencies (float32, head_dim/2 entries; 0 = identity pair)."""
    half = head_dim // 2
    inv = np.zeros(half, dtype=np.float32)
    if not proportional:
        for i in range(half):
            inv[i] = np.float32(theta ** (-2.0 * i / head_dim))
    else:
        rot = int(np.float32(partial) * np.float32(head_dim))
        rot -= rot % 2
        for i in range(rot // 2):
            inv[i] = np.float32(1.0 / float(np.float32(theta ** (2.0 * i / head_dim))))
    return inv


def rope(x: np.ndarray, pos0: int, inv_freq: np.ndarray) -> np.ndarray:
    """x bf16 [L, nh, hd]; rotates (i, i + hd/2) by (pos0 + row) * inv_freq[i]."""
    L, nh, hd = x.shape
    half = hd // 2
    pos = (pos0 + np.arange(L)).astype(np.float32)
    ang = (pos[:, None] * inv_freq[None, :]).astype(np.float32).astype(np.float64)  # fp32 product
    c = np.cos(ang)[:, None, :]
    s = np.sin(ang)[:, None, :]
    xf = fl(x).astype(np.float64)
    x1, x2 = xf[..., :half], xf[..., half:]
    o1 = x1 * c - x2 * s
    o2 = x1 * s + x2 * c
    return bf(np.concatenate([o1, o2], axis=-1).astype(np.float32))


_BF_C = float(fl(bf([0.044715]))[0])
_BF_K = float(fl(bf([0.7978845608028654]))[0])


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """gelu_pytorch_tanh with each MLX bf16 op's rounding (forward.cc:324-336)."""
    xf = fl(x)
    x2 = fl(bf(xf * xf))
    x3 = fl(bf(xf * x2))
    inner = fl(bf(np.float32(_BF_C) * x3))
    inner = fl(bf(inner + xf))
    inner = fl(bf(np.float32(_BF_K) * inner))
    t = fl(bf(np.tanh(inner.astype(np.float64)).astype(np.float32)))
    half_x = fl(bf(np.float32(0.5) * xf))
    one_t = fl(bf(np.float32(1.0) + t))
    return bf(half_x * one_t)


def softcap(logits: np.ndarray, cap: float) -> np.ndarray:
    """cap * tanh(logits / cap), every op in bf16 (forward.cc:154-160)."""
    c = np.float32(fl(bf(cap)))
    d = fl(bf(fl(logits) / c))
    t = fl(bf(np.tanh(d.astype(np.float64)).astype(np.float32)))
    return bf(t * c)


def greedy(logits: np.ndarray) -> Tuple[int, float, bool]:
    """Host scan: first max wins, near_tie = top1 - top2 < 0.5 (forward.cc:162-189)."""
    v = fl(logits).reshape(-1)
    arg = int(np.argmax(v))
    top1 = float(v[arg])
    if v.size > 1:
        top2 = float(np.partition(v, -2)[-2])
    else:
        top2 = -math.inf
    return arg, top1, (top1 - top2) < 0.5


def top_k(logits: np.ndarray, k: int = 8) -> Tuple[np.ndarray, np.ndarray]:
    v = fl(logits).reshape(-1)
    idx = np.argsort(-v, kind="stable")[:k]
    return idx.astype(np.uint32), v[idx]


# ----------------------------------------------------------------------------- KV

class LocalRing:
    """One sliding layer's ring [window + 8, nkv, hd] (kv_cache.cc:134-265)."""

    def __init__(self, window: int, nkv: int, hd: int):
        self.window = window
        self.cap = window + GAMMA_MAX
        self.k = np.zeros((self.cap, nkv, hd), dtype=np.uint16)
        self.v = np.zeros((self.cap, nkv, hd), dtype=np.uint16)
        self.committed = 0

    def slot_for(self, pos: int) -> int:
        return pos % self.cap

    def _write(self, buf, upd, start_slot, n):
        first = min(n, self.cap - start_slot)
        buf[start_slot:start_slot + first] = upd[:first]
        if n > first:
            buf[0:n - first] = upd[first:n]

    def append_committed(self, k: np.ndarray, v: np.ndarray):
        n = k.shape[0]
        written = 0
        while written < n:
            start = self.committed
            take = min(self.cap, n - written)
            self.committed += take
            self._write(self.k, k[written:written + take], self.slot_for(start), take)
            self._write(self.v, v[written:written + take], self.slot_for(start), take)
            written += take

    def read_window(self, buf: np.ndarray, window: int) -> np.ndarray:
        n = min(window, self.committed)
        idx = np.arange(self.committed - n, self.committed) % self.cap
        return buf[idx]

    def nbytes(self) -> int:
        return self.k.nbytes * 2


class GlobalCache:
    """One global layer's linear cache grown by 256-token steps (kv_cache.cc:271-347)."""

    def __init__(self, nkv: int, hd: int):
        self.nkv, self.hd = nkv, hd
        self.k = np.zeros((0, nkv, hd), dtype=np.uint16)
        self.v = np.zeros((0, nkv, hd), dtype=np.uint16)
        self.committed = 0

    def capacity(self) -> int:
        return self.k.shape[0]

    def append(self, k: np.ndarray, v: np.ndarray):
        n = k.shape[0]
        start = self.committed
        self.committed += n
        need = -(-self.committed // GLOBAL_STEP) * GLOBAL_STEP
        if need > self.capacity():
            gk = np.zeros((need, self.nkv, self.hd), dtype=np.uint16)
            gv = np.zeros((need, self.nkv, self.hd), dtype=np.uint16)
            gk[:self.capacity()] = self.k
            gv[:self.capacity()] = self.v
            self.k, self.v = gk, gv
        self.k[start:start + n] = k
        self.v[start:start + n] = v

    def nbytes(self) -> int:
        return self.k.nbytes * 2


# ----------------------------------------------------------------------------- model

class OracleModel:
    def __init__(self, geo: Geometry, tensors: Dict[str, np.ndarray], nthreads: int = 0,
                 sdpa_mode: int = 0):
        self.geo = geo
        self.t = tensors
        self.nt = nthreads
        self.sdpa_mode = sdpa_mode
        self.inv_local = rope_inv_freq(geo.head_dim_local, geo.rope_theta_local, False, 0.0)
        self.inv_global = rope_inv_freq(geo.head_dim_global, geo.rope_theta_global, True,
                                        geo.partial_rotary_factor_global)
        self.embed_scale = bf(math.sqrt(geo.hidden_size))  # fp32 sqrt then bf16 constant
        # Layer kind from the weight schema (v_proj presence), checked against geometry.
        for i in range(geo.num_hidden_layers):
            has_v = f"language_model.model.layers.{i}.self_attn.v_proj.weight" in tensors
            if (0 if has_v else 1) != geo.layer_types[i]:
                raise ValueError(f"layer {i} weight schema disagrees with geometry layer_types")

    # -- helpers
    def _w(self, name):
        return self.t["language_model.model." + name]

    def _proj(self, x, base):
        return qmm(x, self._w(base + ".weight"), self._w(base + ".scales"),
                   self._w(base + ".biases"), self.nt)

    def new_kv(self):
        g = self.geo
        local, glob = [], []
        for i in range(g.num_hidden_layers):
            if g.layer_types[i] == 0:
                local.append(LocalRing(g.sliding_window, g.num_kv_heads_local, g.head_dim_local))
            else:
                glob.append(GlobalCache(g.num_kv_heads_global, g.head_dim_global))
        return {"local": local, "global": glob, "offset": 0, "last_token": 0}

    def _cache_ref(self, layer):
        kinds = self.geo.layer_types[:layer]
        kind = self.geo.layer_types[layer]
        return kind, sum(1 for k in kinds if k == kind)

    def embed(self, ids: np.ndarray) -> np.ndarray:
        w = self._w("embed_tokens.weight")[ids]
        s = fl(self._w("embed_tokens.scales")[ids])
        b = fl(self._w("embed_tokens.biases")[ids])
        L, K8 = w.shape
        codes = np.zeros((L, K8 * 8), dtype=np.float32)
        for i in range(8):
            codes[:, i::8] = ((w >> np.uint32(4 * i)) & np.uint32(0xF)).astype(np.float32)
        g = codes.reshape(L, -1, 64)
        deq = bf((g * s[:, :, None] + b[:, :, None]).reshape(L, -1))  # dequantize -> bf16
        return bf(fl(deq) * fl(self.embed_scale))

    def attention(self, x: np.ndarray, layer: int, kv, offset: int) -> np.ndarray:
        g = self.geo
        kind, j = self._cache_ref(layer)
        hd, nkv, nh = g.head_dim(layer), g.n_kv(layer), g.num_attention_heads
        L = x.shape[0]
        a = f"layers.{layer}.self_attn."
        eps = g.rms_norm_eps
        q = self._proj(x, a + "q_proj").reshape(L, nh, hd)
        q = rms_norm(q, self._w(a + "q_norm.weight"), eps)
        k_raw = self._proj(x, a + "k_proj")
        k = rms_norm(k_raw.reshape(L, nkv, hd), self._w(a + "k_norm.weight"), eps)
        vv = k_raw if kind == 1 else self._proj(x, a + "v_proj")
        v = rms_norm(vv.reshape(L, nkv, hd), None, eps)
        inv = self.inv_local if kind == 0 else self.inv_global
        q = rope(q, offset, inv)
        k = rope(k, offset, inv)
        window = g.sliding_window if kind == 0 else 0
        committed = offset + L
        if kind == 0:
            cache: LocalRing = kv["local"][j]
            if offset > 0 and L > 1:
                pre = min(g.sliding_window, offset)
                k_att = np.concatenate([cache.read_window(cache.k, pre), k])
                v_att = np.concatenate([cache.read_window(cache.v, pre), v])
            cache.append_committed(k, v)
            if offset == 0:
                k_att, v_att = k, v
            elif L == 1:
                n = min(g.sliding_window, cache.committed)
                k_att = cache.read_window(cache.k, n)
                v_att = cache.read_window(cache.v, n)
        else:
            cache: GlobalCache = kv["global"][j]
            cache.append(k, v)
            if offset == 0:
                k_att, v_att = k, v
            else:
                k_att, v_att = cache.k[:committed], cache.v[:committed]
        kv_len = k_att.shape[0]
        o = sdpa(q, k_att, v_att, offset, committed - kv_len, window, 1.0, 0.0,
                 self.sdpa_mode, self.nt)
        return self._proj(o.reshape(L, nh * hd), a + "o_proj")

    def mlp(self, x, layer):
        p = f"layers.{layer}.mlp."
        gate = self._proj(x, p + "gate_proj")
        up = self._proj(x, p + "up_proj")
        act = bf(fl(gelu_tanh(gate)) * fl(up))
        return self._proj(act, p + "down_proj")

    def decoder_layer(self, x, layer, kv, offset, scalar_factor: Optional[float] = None):
        eps = self.geo.rms_norm_eps
        p = f"layers.{layer}."
        h = rms_norm(x, self._w(p + "input_layernorm.weight"), eps)
        h = self.attention(h, layer, kv, offset)
        h = rms_norm(h, self._w(p + "post_attention_layernorm.weight"), eps)
        h = bf(fl(x) + fl(h))
        r = h
        h = rms_norm(h, self._w(p + "pre_feedforward_layernorm.weight"), eps)
        h = self.mlp(h, layer)
        h = rms_norm(h, self._w(p + "post_feedforward_layernorm.weight"), eps)
        h = bf(fl(r) + fl(h))
        sc = self._w(p + "layer_scalar").reshape(-1)[:1]
        if scalar_factor is not None:
            sc = bf(fl(sc) * np.float32(scalar_factor))
        return bf(fl(h) * fl(sc))

    def forward(self, h, kv, offset, fault_layer: Optional[int] = None, factor: float = 1.0):
        for layer in range(self.geo.num_hidden_layers):
            f = factor if layer == fault_layer else None
            h = self.decoder_layer(h, layer, kv, offset, f)
        return rms_norm(h, self._w("norm.weight"), self.geo.rms_norm_eps)

    def logits(self, h_last: np.ndarray) -> np.ndarray:
        """Tied lm_head + bf16 softcap for one row [hidden] -> bf16 [vocab]."""
        lg = qmm(h_last.reshape(1, -1), self._w("embed_tokens.weight"),
                 self._w("embed_tokens.scales"), self._w("embed_tokens.biases"), self.nt)
        return softcap(lg.reshape(-1), self.geo.final_logit_softcapping)

    # -- ABI-level drivers
    def prefill(self, kv, tokens: List[int]):
        assert kv["offset"] == 0
        ids = np.asarray(tokens, dtype=np.int64)
        off = 0
        h = None
        while off < len(ids):
            take = min(PREFILL_CHUNK, len(ids) - off)
            h = self.forward(self.embed(ids[off:off + take]), kv, off)
            off += take
        lg = self.logits(h[-1])
        tok, logit, tie = greedy(lg)
        kv["offset"] = len(ids)
        kv["last_token"] = tok
        return tok, logit, tie, lg

    def decode(self, kv, n_tokens: int = 1, forced: Optional[List[int]] = None):
        """Greedy steps; with ``forced`` the given ids are fed instead (teacher forcing)."""
        out = []
        for step in range(n_tokens):
            tok_in = kv["last_token"] if forced is None else forced[step]
            h = self.forward(self.embed(np.asarray([tok_in])), kv, kv["offset"])
            lg = self.logits(h[-1])
            tok, logit, tie = greedy(lg)
            kv["offset"] += 1
            kv["last_token"] = tok
            out.append((tok, logit, tie, lg))
        return out


# ----------------------------------------------------------------------------- synthetic models

_U64 = (1 << 64) - 1


def host_threads() -> int:
    """Every core this process may run on (OMP_NUM_THREADS, which torchrun sets to 1,
    does not limit the oracle's explicit thread counts)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def normal_table() -> np.ndarray:
    t = np.empty(65536, dtype=np.float32)
    lib().orc_normal_table(_p(t))
    return t


def synth_q4(seed: int, rows: int, K: int, row0: int = 0, col0: int = 0, K_full: Optional[int] = None,
             ztab: Optional[np.ndarray] = None, nthreads: int = 0):
    """Rows [row0, row0 + rows) x columns [col0, col0 + K) of a synthetic [*, K_full]
    Q4/g64 matrix exactly as the engine's synthetic loader generates them."""
    K_full = K if K_full is None else K_full
    ztab = normal_table() if ztab is None else ztab
    nt = nthreads or host_threads()
    w = np.empty((rows, K // 8), dtype=np.uint32)
    s = np.empty((rows, K // 64), dtype=np.uint16)
    b = np.empty((rows, K // 64), dtype=np.uint16)
    lib().orc_synth_words(seed & _U64, rows, K // 8, K_full // 8, row0, col0 // 8, _p(w), nt)
    lib().orc_synth_sb((seed ^ 0x5151) & _U64, rows, K // 64, K_full // 64, row0, col0 // 64, 0.02, _p(ztab),
                       _p(s), _p(b), nt)
    return w, s, b


def synth_norm(seed: int, n: int, ztab: np.ndarray) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().orc_synth_normal(seed & _U64, n, 1.0, 0.02, _p(ztab), _p(out))
    return out


def synthetic_tensors(geo: Geometry, seed: int) -> Dict[str, np.ndarray]:
    """The checkpoint (mlx-lm names) of the engine's seeded synthetic model at TP = 1,
    restating Model::load_synthetic tag for tag: the tied table, the final norm, then per
    layer the fused [q; k; v] matrix (one tag, rows keyed in that order), o_proj, the
    gate/up matrix interleaved by 16-row tiles (tile 2t = gate rows 16t.., 2t + 1 = up
    rows), down_proj and the seven norm/scalar vectors."""
    ztab = normal_table()
    H, I, V = geo.hidden_size, geo.intermediate_size, geo.vocab_size
    nh = geo.num_attention_heads
    t: Dict[str, np.ndarray] = {}
    pre = "language_model.model."
    tag = (seed * 1000003) & _U64

    def nxt():
        nonlocal tag
        tag = (tag + 1) & _U64
        return tag

    t[pre + "embed_tokens.weight"], t[pre + "embed_tokens.scales"], t[pre + "embed_tokens.biases"] = \
        synth_q4(nxt(), V, H, ztab=ztab)
    t[pre + "norm.weight"] = synth_norm(nxt(), H, ztab)
    for i in range(geo.num_hidden_layers):
        hd, nkv, kind = geo.head_dim(i), geo.n_kv(i), geo.layer_types[i]
        p, a = f"{pre}layers.{i}.", f"{pre}layers.{i}.self_attn."
        qf, kf = nh * hd, nkv * hd
        vf = 0 if (kind == 1 and geo.attention_k_eq_v_global) else kf
        w, s, b = synth_q4(nxt(), qf + kf + vf, H, ztab=ztab)
        parts = [("q_proj", 0, qf), ("k_proj", qf, qf + kf)] + ([("v_proj", qf + kf, qf + kf + vf)] if vf else [])
        for nm, r0, r1 in parts:
            t[a + nm + ".weight"], t[a + nm + ".scales"], t[a + nm + ".biases"] = w[r0:r1], s[r0:r1], b[r0:r1]
        t[a + "o_proj.weight"], t[a + "o_proj.scales"], t[a + "o_proj.biases"] = synth_q4(nxt(), H, qf, ztab=ztab)
        gu = synth_q4(nxt(), 2 * I, H, ztab=ztab)
        for j, nm in enumerate(("gate_proj", "up_proj")):
            for suf, arr in zip((".weight", ".scales", ".biases"), gu):
                cols = arr.shape[1]
                t[p + "mlp." + nm + suf] = np.ascontiguousarray(arr.reshape(I // 16, 2, 16, cols)[:, j].reshape(I, cols))
        del gu
        t[p + "mlp.down_proj.weight"], t[p + "mlp.down_proj.scales"], t[p + "mlp.down_proj.biases"] = \
            synth_q4(nxt(), H, I, ztab=ztab)
        t[a + "q_norm.weight"] = synth_norm(nxt(), hd, ztab)
        t[a + "k_norm.weight"] = synth_norm(nxt(), hd, ztab)
        for nm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                   "post_feedforward_layernorm"):
            t[p + nm + ".weight"] = synth_norm(nxt(), H, ztab)
        t[p + "layer_scalar"] = synth_norm(nxt(), 1, ztab)
    return t


# ----------------------------------------------------------------------------- sampling

_RNG_LIB = None


def rng_lib() -> ctypes.CDLL:
    """The standard library's mt19937_64 / uniform_real_distribution<float> draw."""
    global _RNG_LIB
    if _RNG_LIB is None:
        lib()  # builds both libraries
        L = ctypes.CDLL(os.path.join(_HERE, "liboracle_rng.so"))
        L.orc_mt19937_64_first.argtypes = [ctypes.c_uint64]
        L.orc_mt19937_64_first.restype = ctypes.c_uint64
        L.orc_uniform_float_draw.argtypes = [ctypes.c_uint64, ctypes.c_float]
        L.orc_uniform_float_draw.restype = ctypes.c_float
        _RNG_LIB = L
    return _RNG_LIB


def sample(logits_bits: np.ndarray, temperature: float, top_k: int = 0, top_p: float = 0.0, min_p: float = 0.0,
           seed: int = 0):
    """ForwardPass::sample_stochastic (forward.cc:191-322) over one post-softcap bf16 row,
    in float32 with the reference's sequential sums. Sorts are stable (equal values keep
    index order), which the reference leaves unspecified. Returns (token, logit, u, sz,
    kept, top-8 ids, top-8 values)."""
    f32 = np.float32
    src = fl(np.asarray(logits_bits, dtype=np.uint16).reshape(-1))
    n = src.size
    lg = (src * f32(f32(1.0) / f32(temperature))).astype(f32)
    mx = lg.max()
    probs = np.exp((lg - mx).astype(f32)).astype(f32)
    z = np.cumsum(probs, dtype=f32)[-1]
    if z > 0:
        probs = (probs / z).astype(f32)
    ninf = f32(-np.inf)
    lg = lg.copy()
    if 0.0 < top_p <= 1.0:
        order = np.argsort(-probs, kind="stable")
        cum = np.cumsum(probs[order], dtype=f32)
        reach = np.nonzero(cum >= f32(top_p))[0]
        count = (reach[0] + 1) if reach.size else n
        keep = np.zeros(n, dtype=bool)
        keep[order[:count]] = True
        lg[~keep] = ninf
    if 0.0 < min_p < 1.0:
        thr = f32(min_p) * probs.max()
        lg[probs < thr] = ninf
    if 0 < top_k < n:
        order = np.argsort(-lg, kind="stable")
        keep = np.zeros(n, dtype=bool)
        keep[order[:top_k]] = True
        lg[~keep] = ninf
    fmax = lg.max()
    sp = np.where(lg == ninf, f32(0), np.exp((lg - fmax).astype(f32))).astype(f32)
    cum = np.cumsum(sp, dtype=f32)
    sz = cum[-1]
    u = f32(rng_lib().orc_uniform_float_draw(seed & ((1 << 64) - 1), float(sz)))
    hit = np.nonzero(u <= cum)[0]
    tok = int(hit[0]) if hit.size else n - 1
    top = np.argsort(-src, kind="stable")[:min(8, n)]
    return tok, float(src[tok]), float(u), float(sz), int((lg != ninf).sum()), top, src[top]
