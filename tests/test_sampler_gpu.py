"""The device sampler (hyb_sample_logits, and the sampled ABI calls) against the CPU oracle.

The oracle restates ForwardPass::sample_stochastic (native/hyperion_mlx/src/forward.cc:
191-322) in float32 with the reference's sequential sums and draws through the standard
library's std::mt19937_64 / uniform_real_distribution<float>. The device computes the same
steps with tree-ordered parallel sums; the reference sums 262144 floats one after another,
which carries about 1e-4 relative rounding error, so over a whole unfiltered vocabulary the
two pick the same token only when the draw is that far from a boundary. The tests therefore
require: the same generator draw (u / total equal to float rounding); the same kept set
unless a filter cut sits within 1e-4 of a token; the token of exact (float64) arithmetic
over the kept set unless the draw is within 1e-5 of a boundary; the reference-arithmetic
token wherever the kept set is small (<= 1000 tokens, the serving configurations); and the
top-8 sidecar exactly.
"""
import ctypes

import numpy as np
import pytest

import hyperion_b200 as hb
from hyperion_b200.synth import config0, f32_to_bf16_bits
from tests.conftest import has_gpu

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_gpu(), reason="no CUDA device")]

CONFIGS = [  # temperature, top_k, top_p, min_p
    (1.0, 0, 0.0, 0.0),
    (0.8, 40, 0.95, 0.0),
    (0.7, 0, 0.9, 0.0),
    (1.0, 0, 0.0, 0.05),
    (1.3, 200, 0.0, 0.01),
    (0.5, 1, 0.0, 0.0),
]


def _row(n, seed, scale=2.0):
    x = np.random.default_rng(seed).standard_normal(n).astype(np.float32) * scale
    return f32_to_bf16_bits(30.0 * np.tanh(x / 30.0))


def _device_sample(row_dev, n, cfg, seed):
    import torch
    L = hb.lib()
    res = torch.zeros(ctypes.sizeof(hb.HybSampleResult), dtype=torch.uint8, device="cuda")
    c = hb.HypSamplingConfig(cfg[0], cfg[1], cfg[2], cfg[3], seed)
    hb.check(L.hyb_sample_logits(ctypes.c_void_p(row_dev.data_ptr()), n, ctypes.byref(c), seed,
                                 ctypes.c_void_p(res.data_ptr()), None))
    torch.cuda.synchronize()
    return hb.HybSampleResult.from_buffer_copy(res.cpu().numpy().tobytes())


def _exact(row, cfg, kept_order_count, ret):
    """The draw evaluated in float64 over the first `kept` tokens of the (logit desc, index
    asc) order: the exact-arithmetic token and its distance to the nearest CDF boundary
    (relative to the total)."""
    from oracle import gemma_oracle as go
    lg = go.fl(row).astype(np.float64) / np.float32(cfg[0])
    order = np.argsort(-lg, kind="stable")
    keep = np.zeros(row.size, dtype=bool)
    keep[order[:kept_order_count]] = True
    w = np.where(keep, np.exp(lg - lg.max()), 0.0)
    cum = np.cumsum(w)
    u = ret * cum[-1]
    tok = int(np.searchsorted(cum, u, side="left"))
    gap = min(abs(cum[tok] - u), abs((cum[tok - 1] if tok else 0.0) - u)) / cum[-1]
    return min(tok, row.size - 1), gap, cum[-1]


def _filter_margin(row, cfg):
    """How far the top-p and min-p cuts sit from a token boundary (relative units)."""
    from oracle import gemma_oracle as go
    lg = go.fl(row).astype(np.float64) / np.float32(cfg[0])
    p = np.exp(lg - lg.max())
    p /= p.sum()
    m = 1.0
    if cfg[2] > 0:
        m = min(m, float(np.min(np.abs(np.cumsum(np.sort(p)[::-1]) - cfg[2]))))
    if cfg[3] > 0:
        m = min(m, float(np.min(np.abs(p / p.max() - cfg[3]))))
    return m


@pytest.mark.parametrize("n", [262144, 4097, 1000])
def test_device_sampler_matches_oracle(built_lib, oracle_lib, n):
    from oracle import gemma_oracle as go
    from tests.gpu_util import dev
    row = _row(n, n)
    row_dev = dev(row)
    same_as_ref = filtered = exact_ok = total = 0
    for cfg in CONFIGS:
        margin = _filter_margin(row, cfg)
        for seed in range(40 if n == 262144 else 25):
            s = 1000003 * seed + 17
            r = _device_sample(row_dev, n, cfg, s)
            tok, logit, u, sz, kept, top, topv = go.sample(row, *cfg, seed=s)
            total += 1
            # the draw: the same generator output, so u / total agree to float rounding
            ret = u / sz
            assert abs(r.u / r.total - ret) <= 2e-6 * max(1.0, ret), (cfg, s)
            # the filters keep the same tokens unless a cut is within a hair of a token
            assert r.kept == kept or margin < 1e-4, (cfg, s, r.kept, kept)
            # against exact arithmetic over the device's kept set: equal away from a boundary
            etok, gap, esz = _exact(row, cfg, r.kept, r.u / r.total)
            assert abs(r.total - esz) <= 1e-5 * esz, (r.total, esz)
            assert r.token == etok or gap < 1e-5, (cfg, s, r.token, etok, gap)
            exact_ok += r.token == etok
            # against the reference's own float32 arithmetic: short (filtered) sums agree
            same_as_ref += r.token == tok
            if r.token == tok:
                assert r.logit == logit
            if kept <= 1000:
                filtered += 1
                assert r.token == tok or _exact(row, cfg, kept, ret)[1] < 1e-4, (cfg, s, r.token, tok)
            assert list(r.top_k_ids)[:min(8, n)] == list(top) and r.top_k_count == min(8, n)
            assert np.array_equal(np.asarray(list(r.top_k_values)[:8], dtype=np.float32), topv.astype(np.float32))
    print(f"\nn={n}: exact-arithmetic agreement {exact_ok}/{total}, reference-arithmetic agreement "
          f"{same_as_ref}/{total} ({filtered} draws over <= 1000 kept tokens)")
    assert exact_ok / total >= 0.99


def test_device_sampler_is_deterministic_and_validates(built_lib):
    import torch
    from tests.gpu_util import dev
    row = _row(262144, 5)
    row_dev = dev(row)
    a = _device_sample(row_dev, row.size, (0.9, 50, 0.9, 0.0), 123)
    b = _device_sample(row_dev, row.size, (0.9, 50, 0.9, 0.0), 123)
    assert (a.token, a.u, a.total, a.kept) == (b.token, b.u, b.total, b.kept)
    L = hb.lib()
    res = torch.zeros(ctypes.sizeof(hb.HybSampleResult), dtype=torch.uint8, device="cuda")
    for bad in ((0.0, 0, 0.0, 0.0), (1.0, -1, 0.0, 0.0), (1.0, 0, 1.5, 0.0), (1.0, 0, 0.0, 1.0)):
        c = hb.HypSamplingConfig(*bad, 1)
        st = L.hyb_sample_logits(ctypes.c_void_p(row_dev.data_ptr()), row.size, ctypes.byref(c), 1,
                                 ctypes.c_void_p(res.data_ptr()), None)
        assert st == hb.INVALID_ARGUMENT, bad


def test_sampled_abi_calls_match_oracle_on_engine_logits(built_lib, oracle_lib):
    """hyp_decode_block_sampled / hyp_prefill_chunk_sampled against the oracle sampling the
    engine's own logits of the same step (a greedy clone returns them)."""
    from oracle import gemma_oracle as go
    geo = config0()
    eng = hb.Engine(geo, synthetic_seed=12)
    prompt = np.random.default_rng(4).integers(0, geo.vocab_size, 30).tolist()
    base = eng.new_kv()
    base.prefill(prompt)
    agree = total = 0
    for i, cfg in enumerate(CONFIGS):
        for seed in range(5):
            s = 7919 * seed + i
            a, b = base.clone(), base.clone()
            _, lg = a.decode(1, logits=True)
            f, _ = b.decode(1, sampling=hb.HypSamplingConfig(cfg[0], cfg[1], cfg[2], cfg[3], s))
            tok, logit, u, sz, kept, top, topv = go.sample(lg, *cfg, seed=s)
            total += 1
            agree += f.token_id == tok
            if f.token_id != tok:
                assert _exact(lg, cfg, kept, u / sz)[1] < 1e-4
            assert f.top_k_logprob_count == 8 and list(f.top_k_logprob_ids) == list(top)
            assert b.cursor() == (len(prompt) + 1, f.token_id)  # the sampled token feeds the next step
            a.close()
            b.close()
    # a sampled prefill samples the prompt's last row
    kv = eng.new_kv()
    _, lg = kv.prefill(prompt, logits=True)
    cfg = CONFIGS[1]
    kv2 = eng.new_kv()
    f, _ = kv2.prefill(prompt, sampling=hb.HypSamplingConfig(cfg[0], cfg[1], cfg[2], cfg[3], 99))
    tok = go.sample(lg, *cfg, seed=99)[0]
    o = go.sample(lg, *cfg, seed=99)
    assert f.token_id == tok or _exact(lg, cfg, o[4], o[2] / o[3])[1] < 1e-4
    assert agree / total >= 0.95, (agree, total)
