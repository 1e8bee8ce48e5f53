"""hyperion_b200 - B200-native (sm_100a) engine for Hyperion's decode/prefill hot path.

The product is ``libhyperion_mlx.so``: the reference's 14-function
``hyperion_mlx.h`` C ABI (a drop-in for the Rust ``hyperion-ffi`` crate) plus the
op-level extension ABI of ``hyperion_b200.h``. This module binds both with ctypes
so tests and benchmarks call the library exactly as a C caller would. There is
no Python or CPU fallback: if the library is missing this import fails.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhyperion_mlx.so")

# ---------------------------------------------------------------- status codes
OK, INVALID_ARGUMENT, NOT_FOUND, IO, OOM_GOVERNOR, UNSUPPORTED, INTERNAL, CANCELLED = range(8)
STATUS_NAMES = ["OK", "INVALID_ARGUMENT", "NOT_FOUND", "IO", "OOM_GOVERNOR", "UNSUPPORTED", "INTERNAL",
                "CANCELLED"]
LAYER_SLIDING, LAYER_FULL = 0, 1
TOP_K_LOGPROBS = 8


class HypError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES[status] if 0 <= status < 8 else status}: {message}")
        self.status = status
        self.message = message


# ---------------------------------------------------------------- structs (hyperion_mlx.h)
class HypCanaryInfo(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32), ("mlx_compile_major", ctypes.c_uint32),
        ("mlx_compile_minor", ctypes.c_uint32), ("mlx_compile_patch", ctypes.c_uint32),
        ("macos_major", ctypes.c_uint32), ("macos_minor", ctypes.c_uint32), ("macos_patch", ctypes.c_uint32),
        ("gpu_family", ctypes.c_uint32), ("recommended_working_set_bytes", ctypes.c_uint64),
        ("effective_budget_bytes", ctypes.c_uint64), ("soft_watermark_bytes", ctypes.c_uint64),
        ("mlx_probe_value", ctypes.c_float), ("metallib_probe_value", ctypes.c_float),
        ("mlx_runtime_version", ctypes.c_char * 32), ("gpu_name", ctypes.c_char * 128),
    ]


class HypRopeSpec(ctypes.Structure):
    _fields_ = [("theta", ctypes.c_double), ("has_partial_rotary_factor", ctypes.c_int),
                ("partial_rotary_factor", ctypes.c_float), ("proportional", ctypes.c_int)]


class HypMoeConfig(ctypes.Structure):
    _fields_ = [("num_experts", ctypes.c_uint32), ("top_k", ctypes.c_uint32),
                ("moe_intermediate_size", ctypes.c_uint32)]


class HypGeometryParams(ctypes.Structure):
    _fields_ = [
        ("model_type", ctypes.c_int), ("hidden_size", ctypes.c_uint32), ("intermediate_size", ctypes.c_uint32),
        ("num_hidden_layers", ctypes.c_uint32), ("layer_types", ctypes.POINTER(ctypes.c_int)),
        ("num_attention_heads", ctypes.c_uint32), ("head_dim_local", ctypes.c_uint32),
        ("head_dim_global", ctypes.c_uint32), ("num_kv_heads_local", ctypes.c_uint32),
        ("num_kv_heads_global", ctypes.c_uint32), ("attention_k_eq_v_global", ctypes.c_int),
        ("num_kv_shared_layers", ctypes.c_uint32), ("sliding_window", ctypes.c_uint32),
        ("rope_local", HypRopeSpec), ("rope_global", HypRopeSpec),
        ("final_logit_softcapping", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
        ("attention_bias", ctypes.c_int), ("vocab_size", ctypes.c_uint32),
        ("max_position_embeddings", ctypes.c_uint32), ("tie_word_embeddings", ctypes.c_int),
        ("ple_hidden_per_layer_input", ctypes.c_uint32), ("ple_vocab_per_layer_input", ctypes.c_uint32),
        ("use_double_wide_mlp", ctypes.c_int), ("has_moe", ctypes.c_int), ("moe", HypMoeConfig),
    ]


class HypTokenStream(ctypes.Structure):
    _fields_ = [("tokens", ctypes.POINTER(ctypes.c_uint32)), ("count", ctypes.c_uint32),
                ("is_prompt", ctypes.c_int)]


class HypSamplingConfig(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int32), ("top_p", ctypes.c_float),
                ("min_p", ctypes.c_float), ("seed", ctypes.c_uint64)]


class HybSampleResult(ctypes.Structure):
    _fields_ = [("token", ctypes.c_uint32), ("logit", ctypes.c_float), ("top_k_ids", ctypes.c_uint32 * 8),
                ("top_k_values", ctypes.c_float * 8), ("top_k_count", ctypes.c_uint32), ("kept", ctypes.c_uint32),
                ("u", ctypes.c_float), ("total", ctypes.c_float)]


class HypStepResultFields(ctypes.Structure):
    _fields_ = [
        ("token_id", ctypes.c_uint32), ("logit", ctypes.c_float), ("peak_mlx_bytes", ctypes.c_uint64),
        ("active_mlx_bytes", ctypes.c_uint64), ("phys_footprint_bytes", ctypes.c_uint64),
        ("local_kv_bytes", ctypes.c_uint64), ("global_kv_bytes", ctypes.c_uint64),
        ("local_kv_eval_ms", ctypes.c_float), ("global_kv_eval_ms", ctypes.c_float),
        ("governor_state", ctypes.c_int), ("near_tie_events", ctypes.c_uint32),
        ("top_k_logprob_count", ctypes.c_uint32),
        ("top_k_logprob_ids", ctypes.c_uint32 * TOP_K_LOGPROBS),
        ("top_k_logprob_values", ctypes.c_float * TOP_K_LOGPROBS),
    ]


# The 14 functions of hyperion_mlx.h plus the hyperion_b200.h extensions.
ABI_FUNCTIONS = [
    "hyp_runtime_canary", "hyp_last_error", "hyp_model_create", "hyp_model_free", "hyp_model_load",
    "hyp_kvstate_create", "hyp_kvstate_free", "hyp_prefill_chunk", "hyp_decode_block",
    "hyp_prefill_chunk_sampled", "hyp_decode_block_sampled", "hyp_step_result_create",
    "hyp_step_result_free", "hyp_step_result_fields",
]
EXT_FUNCTIONS = [
    "hyb_build_info", "hyb_quantized_matmul", "hyb_qmv_fused", "hyb_qmv_packed_bytes", "hyb_qmv_pack",
    "hyb_qmv_packed", "hyb_sdpa_decode_scratch_bytes", "hyb_sdpa_decode", "hyb_sdpa_decode_noalloc",
    "hyb_sdpa_decode_fused", "hyb_wait_timeouts", "hyb_nccl_unique_id", "hyb_model_set_tensor_parallel",
    "hyb_sdpa_prefill", "hyb_rms_norm", "hyb_qkv_post", "hyb_model_load_synthetic",
    "hyb_model_set_attention_rounding", "hyb_model_stream", "hyb_decode_batch", "hyb_kvstate_clone", "hyb_qmv_batched",
    "hyb_verify",
    "hyb_kv_copy_layer", "hyb_kv_cursor", "hyb_prefill_logits", "hyb_decode_logits", "hyb_decode_forced",
    "hyb_test_arm_post_append_fault", "hyb_model_set_memory_budget", "hyb_sample_logits",
    "hyb_model_weight_bytes", "hyb_qmv_unpack", "hyb_embed_packed",
]

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load libhyperion_mlx.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m hyperion_b200.build` "
                          "(the CUDA engine has no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P, c = ctypes.c_void_p, ctypes
    S = ctypes.c_int  # HypStatus
    sig = {
        "hyp_runtime_canary": [ctypes.POINTER(HypCanaryInfo)],
        "hyp_last_error": [c.c_char_p, c.c_size_t],
        "hyp_model_create": [ctypes.POINTER(P)],
        "hyp_model_free": [ctypes.POINTER(P)],
        "hyp_model_load": [P, ctypes.POINTER(HypGeometryParams), c.c_char_p],
        "hyp_kvstate_create": [P, ctypes.POINTER(P)],
        "hyp_kvstate_free": [ctypes.POINTER(P)],
        "hyp_prefill_chunk": [P, P, ctypes.POINTER(HypTokenStream), P],
        "hyp_decode_block": [P, P, c.c_uint32, P],
        "hyp_prefill_chunk_sampled": [P, P, ctypes.POINTER(HypTokenStream), ctypes.POINTER(HypSamplingConfig), P],
        "hyp_decode_block_sampled": [P, P, c.c_uint32, ctypes.POINTER(HypSamplingConfig), P],
        "hyp_step_result_create": [ctypes.POINTER(P)],
        "hyp_step_result_free": [ctypes.POINTER(P)],
        "hyp_step_result_fields": [P, ctypes.POINTER(HypStepResultFields)],
        "hyb_build_info": [c.c_char_p, c.c_size_t],
        "hyb_quantized_matmul": [P, P, P, P, P, c.c_int64, c.c_int64, c.c_int64, c.c_int32, c.c_int32, P],
        "hyb_qmv_fused": [P, P, P, P, P, c.c_int64, c.c_int64, c.c_int32, c.c_int32, P, P, P, P, P, c.c_float, P],
        "hyb_qmv_pack": [P, P, P, c.c_int64, c.c_int64, P, P],
        "hyb_qmv_unpack": [P, c.c_int64, c.c_int64, P, P, P, P],
        "hyb_embed_packed": [P, c.c_int64, P, c.c_int64, c.c_int64, c.c_uint16, P, P],
        "hyb_qmv_packed": [P, P, P, c.c_int64, c.c_int64, c.c_int32, c.c_int32, P, P, P, P, P, c.c_float, P],
        "hyb_sdpa_decode": [P, P, P, P, c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32,
                            c.c_float, c.c_float, c.c_int32, P, c.c_size_t, P],
        "hyb_sdpa_decode_fused": [P, c.c_int32, P, P, P, c.c_float, P, P, c.c_int32, c.c_int32, c.c_int32,
                                  c.c_int32, c.c_int32, c.c_int32, c.c_float, c.c_float, c.c_int32, P, P],
        "hyb_wait_timeouts": [c.POINTER(c.c_int64)],
        "hyb_nccl_unique_id": [P],
        "hyb_model_set_tensor_parallel": [P, c.c_int32, c.c_int32, P],
        "hyb_sdpa_decode_noalloc": [P, P, P, P, c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32,
                                    c.c_int32, c.c_float, c.c_float, c.c_int32, P],
        "hyb_sdpa_prefill": [P, P, P, P, c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32,
                             c.c_int32, c.c_int32, c.c_float, c.c_float, c.c_int32, P],
        "hyb_rms_norm": [P, P, P, c.c_int32, c.c_int32, c.c_float, P],
        "hyb_qkv_post": [P, c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32, P, P, P,
                         c.c_int32, c.c_float, P, P, P, P, P, c.c_int32, c.c_int32, P],
        "hyb_model_load_synthetic": [P, ctypes.POINTER(HypGeometryParams), c.c_uint64],
        "hyb_model_set_attention_rounding": [P, c.c_int32],
        "hyb_kvstate_clone": [P, P, c.c_uint32, ctypes.POINTER(P)],
        "hyb_qmv_batched": [P, c.c_int32, c.c_int64, P, P, c.c_int64, c.c_int64, c.c_int64, c.c_int32, P],
        "hyb_decode_batch": [P, ctypes.POINTER(P), c.c_uint32, ctypes.POINTER(c.c_uint32), ctypes.POINTER(c.c_float)],
        "hyb_verify": [P, P, ctypes.POINTER(c.c_uint32), c.c_uint32, ctypes.POINTER(c.c_uint32),
                       ctypes.POINTER(c.c_float), ctypes.POINTER(c.c_uint32)],
        "hyb_model_stream": [P, ctypes.POINTER(P)],
        "hyb_kv_copy_layer": [P, P, c.c_uint32, c.c_int32, P, ctypes.POINTER(c.c_uint32)],
        "hyb_kv_cursor": [P, ctypes.POINTER(c.c_uint32), ctypes.POINTER(c.c_uint32)],
        "hyb_prefill_logits": [P, P, ctypes.POINTER(HypTokenStream), P, P],
        "hyb_decode_logits": [P, P, P, P],
        "hyb_decode_forced": [P, P, c.c_uint32, P, P],
        "hyb_test_arm_post_append_fault": [],
        "hyb_model_set_memory_budget": [P, c.c_uint64],
        "hyb_model_weight_bytes": [P, c.POINTER(c.c_uint64), c.POINTER(c.c_uint64), c.POINTER(c.c_uint64)],
        "hyb_sample_logits": [P, c.c_int32, ctypes.POINTER(HypSamplingConfig), c.c_uint64, P, P],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = S
    L.hyb_sdpa_decode_scratch_bytes.argtypes = [c.c_int32, c.c_int32, c.c_int32, c.c_int32]
    L.hyb_sdpa_decode_scratch_bytes.restype = c.c_size_t
    L.hyb_qmv_packed_bytes.argtypes = [c.c_int64, c.c_int64]
    L.hyb_qmv_packed_bytes.restype = c.c_size_t
    _lib = L
    return L


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().hyp_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def tp_shard_check(geo, tp: int) -> Optional[str]:
    """Why `geo` cannot be split over `tp` ranks (the engine's rule), or None if it can:
    heads and KV heads split evenly, MLP rows in 16-row tiles and 64-wide K groups, the
    per-rank attention width in 64-wide groups, and the vocabulary evenly."""
    if tp < 1 or tp > 8:
        return "tensor parallel size must be 1..8"
    if tp == 1:
        return None
    h, i, v = geo.num_attention_heads, geo.intermediate_size, geo.vocab_size
    if h % tp or i % (16 * tp) or v % tp or (i // tp) % 64:
        return "heads, MLP rows and vocabulary must split evenly over the ranks"
    if (h // tp) * geo.head_dim_local % 64 or (h // tp) * geo.head_dim_global % 64:
        return "the per-rank attention width must be a multiple of 64"
    if geo.num_kv_heads_local % tp or geo.num_kv_heads_global % tp:
        return "KV heads must split evenly over the ranks"
    return None


def nccl_unique_id() -> bytes:
    """128-byte NCCL unique id for hyb_model_set_tensor_parallel (created on rank 0)."""
    buf = ctypes.create_string_buffer(128)
    check(lib().hyb_nccl_unique_id(buf))
    return buf.raw


def check(status: int) -> None:
    if status != OK:
        raise HypError(status, last_error())


# ---------------------------------------------------------------- geometry helpers
def geometry_params(geo) -> HypGeometryParams:
    """Build HypGeometryParams from a hyperion_b200.synth.Geometry (keeps the layer array alive)."""
    arr = (ctypes.c_int * len(geo.layer_types))(*geo.layer_types)
    p = HypGeometryParams()
    p.model_type = geo.model_type
    p.hidden_size = geo.hidden_size
    p.intermediate_size = geo.intermediate_size
    p.num_hidden_layers = geo.num_hidden_layers
    p.layer_types = ctypes.cast(arr, ctypes.POINTER(ctypes.c_int))
    p.num_attention_heads = geo.num_attention_heads
    p.head_dim_local = geo.head_dim_local
    p.head_dim_global = geo.head_dim_global
    p.num_kv_heads_local = geo.num_kv_heads_local
    p.num_kv_heads_global = geo.num_kv_heads_global
    p.attention_k_eq_v_global = geo.attention_k_eq_v_global
    p.num_kv_shared_layers = 0
    p.sliding_window = geo.sliding_window
    p.rope_local = HypRopeSpec(geo.rope_theta_local, 0, 0.0, 0)
    p.rope_global = HypRopeSpec(geo.rope_theta_global, 1, geo.partial_rotary_factor_global, 1)
    p.final_logit_softcapping = geo.final_logit_softcapping
    p.rms_norm_eps = geo.rms_norm_eps
    p.attention_bias = 0
    p.vocab_size = geo.vocab_size
    p.max_position_embeddings = geo.max_position_embeddings
    p.tie_word_embeddings = 1
    p._layer_arr = arr  # keep alive
    return p


# ---------------------------------------------------------------- engine wrapper
class Engine:
    """Owns a HypModel; thin Pythonic layer over the C ABI (used by tests and bench)."""

    def __init__(self, geo, weights_dir: Optional[str] = None, synthetic_seed: Optional[int] = None,
                 tp: Optional[tuple] = None):
        """tp = (rank, size, unique_id bytes) loads this rank's tensor-parallel shard."""
        L = lib()
        self.geo = geo
        self.vocab = geo.vocab_size
        self._model = ctypes.c_void_p()
        check(L.hyp_model_create(ctypes.byref(self._model)))
        self._params = geometry_params(geo)
        if tp is not None:
            rank, size, uid = tp
            buf = ctypes.create_string_buffer(bytes(uid), 128)
            st = L.hyb_model_set_tensor_parallel(self._model, rank, size, buf)
            if st != OK:
                msg = last_error()
                L.hyp_model_free(ctypes.byref(self._model))
                raise HypError(st, msg)
        if synthetic_seed is not None:
            st = L.hyb_model_load_synthetic(self._model, ctypes.byref(self._params), synthetic_seed)
        else:
            st = L.hyp_model_load(self._model, ctypes.byref(self._params), weights_dir.encode())
        if st != OK:
            msg = last_error()
            L.hyp_model_free(ctypes.byref(self._model))
            raise HypError(st, msg)
        self._result = ctypes.c_void_p()
        check(L.hyp_step_result_create(ctypes.byref(self._result)))

    def close(self):
        L = lib()
        if self._result:
            L.hyp_step_result_free(ctypes.byref(self._result))
        if self._model:
            L.hyp_model_free(ctypes.byref(self._model))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._model

    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(lib().hyb_model_stream(self._model, ctypes.byref(s)))
        return s.value or 0

    def set_attention_rounding(self, mode: int) -> None:
        check(lib().hyb_model_set_attention_rounding(self._model, mode))

    def set_memory_budget(self, nbytes: int) -> None:
        """Device-byte ceiling checked by every call's admission (0 = free memory only)."""
        check(lib().hyb_model_set_memory_budget(self._model, nbytes))

    def weight_bytes(self) -> dict:
        """Device bytes of the weights: resident, algorithmic (codes + scales + biases)
        and the MLX-layout unpack scratch (hyb_model_weight_bytes)."""
        r, a, s = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        check(lib().hyb_model_weight_bytes(self._model, ctypes.byref(r), ctypes.byref(a), ctypes.byref(s)))
        return {"resident": r.value, "algorithmic": a.value, "scratch": s.value}

    def decode_batch(self, kvs: Sequence["KvState"]):
        """One greedy step of every state in `kvs` together (hyb_decode_batch):
        returns (tokens, post-softcap logits), one per state."""
        n = len(kvs)
        arr = (ctypes.c_void_p * n)(*[k._kv.value for k in kvs])
        toks = (ctypes.c_uint32 * n)()
        logs = (ctypes.c_float * n)()
        check(lib().hyb_decode_batch(self._model, arr, n, toks, logs))
        return list(toks), list(logs)

    def new_kv(self) -> "KvState":
        return KvState(self)

    def fields(self) -> HypStepResultFields:
        f = HypStepResultFields()
        check(lib().hyp_step_result_fields(self._result, ctypes.byref(f)))
        return f


class KvState:
    def __init__(self, eng: Engine):
        self.eng = eng
        self._kv = ctypes.c_void_p()
        check(lib().hyp_kvstate_create(eng.handle, ctypes.byref(self._kv)))

    def clone(self, last_token: Optional[int] = None) -> "KvState":
        """A copy of this state (hyb_kvstate_clone) whose next input is `last_token`."""
        k = KvState.__new__(KvState)
        k.eng = self.eng
        k._kv = ctypes.c_void_p()
        check(lib().hyb_kvstate_clone(self.eng.handle, self._kv, 0xFFFFFFFF if last_token is None else last_token,
                                      ctypes.byref(k._kv)))
        return k

    def verify(self, draft: Sequence[int]):
        """Greedy speculative verify of `draft` (1..8 tokens, hyb_verify): returns
        (accepted, tokens, post-softcap logits) with len(draft) + 1 greedy samples; the
        state advances by accepted + 1 tokens."""
        n = len(draft)
        d = (ctypes.c_uint32 * max(n, 1))(*draft)
        toks = (ctypes.c_uint32 * (n + 1))()
        logs = (ctypes.c_float * (n + 1))()
        acc = ctypes.c_uint32()
        check(lib().hyb_verify(self.eng.handle, self._kv, d, n, toks, logs, ctypes.byref(acc)))
        return acc.value, list(toks), list(logs)

    def close(self):
        if self._kv:
            lib().hyp_kvstate_free(ctypes.byref(self._kv))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._kv

    def _logits_buf(self, want: bool):
        if not want:
            return None, None
        import numpy as np
        buf = np.empty(self.eng.vocab, dtype=np.uint16)
        return buf, buf.ctypes.data_as(ctypes.c_void_p)

    def prefill(self, tokens: Sequence[int], logits: bool = False, sampling: Optional[HypSamplingConfig] = None):
        arr = (ctypes.c_uint32 * len(tokens))(*tokens)
        ts = HypTokenStream(ctypes.cast(arr, ctypes.POINTER(ctypes.c_uint32)), len(tokens), 1)
        buf, ptr = self._logits_buf(logits)
        L = lib()
        if sampling is not None:
            check(L.hyp_prefill_chunk_sampled(self.eng.handle, self._kv, ctypes.byref(ts), ctypes.byref(sampling),
                                              self.eng._result))
        elif logits:
            check(L.hyb_prefill_logits(self.eng.handle, self._kv, ctypes.byref(ts), self.eng._result, ptr))
        else:
            check(L.hyp_prefill_chunk(self.eng.handle, self._kv, ctypes.byref(ts), self.eng._result))
        return self.eng.fields(), buf

    def decode(self, n: int = 1, logits: bool = False, forced: Optional[int] = None,
               sampling: Optional[HypSamplingConfig] = None):
        L = lib()
        buf, ptr = self._logits_buf(logits)
        if forced is not None:
            check(L.hyb_decode_forced(self.eng.handle, self._kv, forced, self.eng._result, ptr))
        elif sampling is not None:
            check(L.hyp_decode_block_sampled(self.eng.handle, self._kv, n, ctypes.byref(sampling), self.eng._result))
        elif logits:
            assert n == 1
            check(L.hyb_decode_logits(self.eng.handle, self._kv, self.eng._result, ptr))
        else:
            check(L.hyp_decode_block(self.eng.handle, self._kv, n, self.eng._result))
        return self.eng.fields(), buf

    def cursor(self):
        o, t = ctypes.c_uint32(), ctypes.c_uint32()
        check(lib().hyb_kv_cursor(self._kv, ctypes.byref(o), ctypes.byref(t)))
        return o.value, t.value

    def copy_layer(self, layer: int, which: int):
        import numpy as np
        rows = ctypes.c_uint32(0)
        check(lib().hyb_kv_copy_layer(self.eng.handle, self._kv, layer, which, None, ctypes.byref(rows)))
        g = self.eng.geo
        row = g.n_kv(layer) * g.head_dim(layer)
        out = np.empty((rows.value, g.n_kv(layer), g.head_dim(layer)), dtype=np.uint16)
        n = ctypes.c_uint32(rows.value)
        check(lib().hyb_kv_copy_layer(self.eng.handle, self._kv, layer, which,
                                      out.ctypes.data_as(ctypes.c_void_p), ctypes.byref(n)))
        assert out.size == rows.value * row
        return out
