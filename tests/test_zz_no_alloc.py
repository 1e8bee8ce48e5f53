"""hyb_sdpa_decode_noalloc: decode attention for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc (a host runtime that owns the whole device pool,
or a per-token loop that cannot take the synchronization an allocation may cause).
This entry point gives them the split-K decode attention with its scratch in a fixed
8 MiB device array instead of a caller buffer. The test calls it through the C ABI
(ctypes on libhyperion_mlx.so) twice in a row and checks each result against the
scratch-taking hyb_sdpa_decode on the same inputs, within the tolerance the other
attention tests use. The file name sorts last so that a run stopping at the first
failure has run every other test before this one; the test also passes alone in a
fresh process (the first call performs the per-device set-up).
"""
import ctypes

import numpy as np
import pytest

from hyperion_b200.synth import f32_to_bf16_bits
from tests.conftest import has_gpu

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_gpu(), reason="no CUDA device")]

REL_L2_BF16 = 2e-3  # the bound the other attention tests use


def _case(H, Hkv, hd, cap, last_pos, n_keys, seed):
    import torch
    from tests.gpu_util import dev
    rng = np.random.default_rng(seed)
    q = dev(f32_to_bf16_bits(rng.standard_normal((H, hd), dtype=np.float32)))
    k = dev(f32_to_bf16_bits(rng.standard_normal((cap, Hkv, hd), dtype=np.float32)))
    v = dev(f32_to_bf16_bits(rng.standard_normal((cap, Hkv, hd), dtype=np.float32)))
    return q, k, v


def _rel_l2(a, b):
    a = a.float().cpu().numpy().astype(np.float64)
    b = b.float().cpu().numpy().astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_noalloc_decode_matches_scratch_version_twice(built_lib):
    import torch
    import hyperion_b200 as hb
    L = built_lib
    P = ctypes.c_void_p
    stream = P(torch.cuda.current_stream().cuda_stream)
    # calls in a row: a wrapped sliding-window ring, then a global cache, then a call with
    # few heads of another head_dim and few keys, which follows calls that left the shared
    # buffer full of nonzero partials (its counters must be cleared, its stale scores unread)
    cases = [(16, 8, 256, 1032, 2999, 1024, 1 / 16.0, 0), (32, 16, 128, 4352, 4099, 4100, 1 / 11.3, 1),
             (4, 2, 64, 512, 300, 301, 1 / 8.0, 2)]
    for (H, Hkv, hd, cap, last_pos, n_keys, scale, seed) in cases:
        q, k, v = _case(H, Hkv, hd, cap, last_pos, n_keys, seed)
        # reference result: the same kernel with a caller-provided, freshly zeroed scratch
        nbytes = L.hyb_sdpa_decode_scratch_bytes(H, Hkv, hd, n_keys)
        scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        ref = torch.empty_like(q)
        hb.check(L.hyb_sdpa_decode(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(ref.data_ptr()), H, Hkv,
                                   hd, cap, last_pos, n_keys, scale, 0.0, 0, P(scratch.data_ptr()), nbytes, stream))
        out = torch.empty_like(q)
        hb.check(L.hyb_sdpa_decode_noalloc(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(out.data_ptr()), H,
                                           Hkv, hd, cap, last_pos, n_keys, scale, 0.0, 0, stream))
        torch.cuda.synchronize()
        assert _rel_l2(out, ref) <= REL_L2_BF16
        assert torch.equal(out, ref)  # same kernel, same split order: identical bits


def test_noalloc_decode_rejected_call_leaves_next_call_intact(built_lib):
    """A call refused for its shape queues nothing, so the next call's result is unchanged."""
    import torch
    import hyperion_b200 as hb
    L = built_lib
    P = ctypes.c_void_p
    stream = P(torch.cuda.current_stream().cuda_stream)
    H, Hkv, hd, cap, last_pos, n_keys = 8, 2, 128, 1024, 700, 701
    q, k, v = _case(H, Hkv, hd, cap, last_pos, n_keys, 3)
    nbytes = L.hyb_sdpa_decode_scratch_bytes(H, Hkv, hd, n_keys)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    ref = torch.empty_like(q)
    hb.check(L.hyb_sdpa_decode(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(ref.data_ptr()), H, Hkv, hd,
                               cap, last_pos, n_keys, 1.0, 0.0, 0, P(scratch.data_ptr()), nbytes, stream))
    # 16 query heads over one KV head: past the argument checks, refused by the kernel's shape
    # checks (GQA group above 8), which run before the shared buffer is touched
    bad = L.hyb_sdpa_decode_noalloc(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(ref.data_ptr()), 16, 1, 64,
                                    cap, last_pos, n_keys, 1.0, 0.0, 0, stream)
    assert bad == hb.INVALID_ARGUMENT and "GQA" in hb.last_error()
    out = torch.empty_like(q)
    hb.check(L.hyb_sdpa_decode_noalloc(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(out.data_ptr()), H, Hkv,
                                       hd, cap, last_pos, n_keys, 1.0, 0.0, 0, stream))
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_noalloc_decode_rejects_requests_above_the_fixed_buffer(built_lib):
    import torch
    import hyperion_b200 as hb
    L = built_lib
    P = ctypes.c_void_p
    # 64 heads over 8 KV heads, head_dim 128, 32768 keys: needs ~10 MiB of scratch
    H, Hkv, hd, n_keys = 64, 8, 128, 32768
    assert L.hyb_sdpa_decode_scratch_bytes(H, Hkv, hd, n_keys) > 8 * 2 ** 20
    q = torch.zeros((H, hd), dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros((n_keys, Hkv, hd), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(q)
    st = L.hyb_sdpa_decode_noalloc(P(q.data_ptr()), P(kc.data_ptr()), P(kc.data_ptr()), P(out.data_ptr()), H, Hkv,
                                   hd, n_keys, n_keys - 1, n_keys, 1.0, 0.0, 0,
                                   P(torch.cuda.current_stream().cuda_stream))
    assert st == hb.INVALID_ARGUMENT
    assert "8 MiB" in hb.last_error()
