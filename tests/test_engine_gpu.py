"""End-to-end parity of the CUDA engine through the 14-function ABI.

The engine loads seeded synthetic checkpoints (written as mlx-lm style
safetensors, read by the C++ loader), runs prefill + greedy decode, and is
compared with the oracle running the reference's op graph on the same packed
weights: tokens, post-softcap logits, and the bytes of the KV caches.
"""
import ctypes

import numpy as np
import pytest

import hyperion_b200 as hb
from hyperion_b200.synth import bf16_bits_to_f32, config0, config3, tiny_fixture_geometry, write_checkpoint, Geometry
from tests.conftest import has_gpu
from tests.gpu_util import max_ulp, rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_gpu(), reason="no CUDA device")]


def _setup(tmp_path, geo, seed):
    from oracle import gemma_oracle as go
    d = tmp_path / f"ckpt{seed}"
    t = write_checkpoint(geo, str(d), seed=seed)
    return hb.Engine(geo, weights_dir=str(d)), go.OracleModel(geo, t)


def _prompt(geo, n, seed):
    return np.random.default_rng(seed).integers(0, geo.vocab_size, n).tolist()


def test_canary_on_gpu(built_lib):
    info = hb.HypCanaryInfo()
    hb.check(built_lib.hyp_runtime_canary(ctypes.byref(info)))
    assert info.abi_version == 3
    assert info.mlx_probe_value == 4.0 and info.metallib_probe_value == 42.0
    assert info.gpu_family >= 100
    assert info.recommended_working_set_bytes > 100 * 2 ** 30


@pytest.mark.parametrize("geo_name", ["cfg0", "cfg3_2layers"])
def test_weights_resident_once(built_lib, geo_name):
    """Every quantised matrix is held once, in the packed layout: resident weight bytes are
    the algorithmic size (codes + scales + biases) plus norms, and the MLX-layout scratch the
    prefill GEMM unpacks into is one projection (or one lm_head slice)."""
    geo = {"cfg0": config0(), "cfg3_2layers": config3(2)}[geo_name]
    eng = hb.Engine(geo, synthetic_seed=5)
    wb = eng.weight_bytes()
    H, V = geo.hidden_size, geo.vocab_size
    assert wb["algorithmic"] >= V * H * 9 // 16
    small = geo.num_hidden_layers * (6 * H + 2 * 512 + 2) * 2 + 2 * H + 4 * 1024  # norms, RoPE
    pad = (4 * geo.num_hidden_layers + 1) * 15 * max(H, geo.intermediate_size) * 9 // 16  # 16-row blocks
    assert wb["algorithmic"] <= wb["resident"] <= wb["algorithmic"] + pad + small, wb
    assert wb["scratch"] <= 0.6 * wb["algorithmic"], wb
    if geo_name == "cfg3_2layers":
        assert wb["scratch"] <= 80 * 2 ** 20, wb  # one 30720 x 3840 gate/up matrix


def _teacher_forced(eng, orc, prompt, steps):
    """Run the engine greedily; the oracle consumes the engine's token stream.
    Returns (token agreement per step, logits rel-L2 per step incl. prefill)."""
    kv = eng.new_kv()
    f, lg = kv.prefill(prompt, logits=True)
    okv = orc.new_kv()
    otok, _, _, olg = orc.prefill(okv, prompt)
    agree, rels = [f.token_id == otok], [rel_l2(lg, olg)]
    prev = f.token_id
    for _ in range(steps):
        f, lg = kv.decode(1, logits=True)
        (o_tok, _, _, o_lg), = orc.decode(okv, 1, forced=[prev])
        agree.append(f.token_id == o_tok)
        rels.append(rel_l2(lg, o_lg))
        prev = f.token_id
    off, last = kv.cursor()
    assert off == len(prompt) + steps and last == prev
    return np.asarray(agree), np.asarray(rels)


@pytest.mark.parametrize("geo_name", ["cfg0", "tiny", "cfg3_2layers"])
def test_decode_step_stagewise(built_lib, oracle_lib, tmp_path, geo_name):
    """One decode step replayed stage by stage through the op-level ABI, each stage
    fed the oracle's own input, exactly as the engine wires the fused kernels:
    norm-prologue qkv qmv -> QK-norm/RoPE/cache write -> split-K attention over the
    ring or global cache -> o_proj -> residual+norm prologue gate/up qmv with the
    GeGLU epilogue -> down. Every stage must sit within the per-op bound. cfg3_2layers
    runs the 12B shapes (hd 256, 16/8 heads, hidden 3840, MLP 15360) on one sliding and
    one global layer of the seeded synthetic model."""
    import torch
    from hyperion_b200 import ops
    from oracle import gemma_oracle as go
    from tests.gpu_util import dev, host
    if geo_name == "cfg3_2layers":
        geo = config3(2)
        t = go.synthetic_tensors(geo, 7)
    else:
        geo = config0() if geo_name == "cfg0" else tiny_fixture_geometry()
        t = write_checkpoint(geo, str(tmp_path / "w"), seed=7)
    orc = go.OracleModel(geo, t, nthreads=go.host_threads())
    prompt = _prompt(geo, 32, 7)
    okv = orc.new_kv()
    tok = orc.prefill(okv, prompt)[0]
    W = lambda n: t["language_model.model." + n]
    H, I, nh, eps, pos = geo.hidden_size, geo.intermediate_size, geo.num_attention_heads, 1e-6, len(prompt)
    h = orc.embed(np.asarray([tok]))[0]
    li = gi = 0

    def close(got, want, bound=5e-4):
        assert rel_l2(got, want) <= bound and (got == want).mean() >= 0.95

    for layer, kind in enumerate(geo.layer_types):
        p, a = f"layers.{layer}.", f"layers.{layer}.self_attn."
        hd, nkv = geo.head_dim(layer), geo.n_kv(layer)
        names = [a + "q_proj", a + "k_proj"] + ([a + "v_proj"] if kind == 0 else [])
        Wq, Sq, Bq = (np.concatenate([W(n + suf) for n in names]) for suf in (".weight", ".scales", ".biases"))
        xn = go.rms_norm(h.reshape(1, H), W(p + "input_layernorm.weight"), eps)
        want_qkv = go.qmm(xn, Wq, Sq, Bq).reshape(-1)
        got_qkv = host(ops.qmv_fused(dev(h), dev(Wq), dev(Sq), dev(Bq), prologue=1,
                                     norm_w=dev(W(p + "input_layernorm.weight"))))
        close(got_qkv, want_qkv)
        inv = orc.inv_local if kind == 0 else orc.inv_global
        q_o = go.rope(go.rms_norm(want_qkv[:nh * hd].reshape(1, nh, hd), W(a + "q_norm.weight"), eps), pos, inv)
        kraw = want_qkv[nh * hd:(nh + nkv) * hd].reshape(1, nkv, hd)
        k_o = go.rope(go.rms_norm(kraw, W(a + "k_norm.weight"), eps), pos, inv)
        vsrc = kraw if kind == 1 else want_qkv[(nh + nkv) * hd:].reshape(1, nkv, hd)
        v_o = go.rms_norm(vsrc, None, eps)
        qg, kg, vg = ops.qkv_post(dev(want_qkv.reshape(1, -1)), nh, nkv, hd, kind == 1, dev(W(a + "q_norm.weight")),
                                  dev(W(a + "k_norm.weight")), dev(inv), pos)
        for got, want in ((qg, q_o), (kg, k_o), (vg, v_o)):
            close(host(got).reshape(-1), want.reshape(-1))
        if kind == 0:
            c = okv["local"][li]
            kc, vc, cap = c.k.copy(), c.v.copy(), c.cap
            li += 1
            n_keys = min(geo.sliding_window, pos + 1)
        else:
            c = okv["global"][gi]
            kc, vc, cap = c.k.copy(), c.v.copy(), c.capacity()
            gi += 1
            n_keys = pos + 1
        kc[pos % cap], vc[pos % cap] = k_o[0], v_o[0]
        ps = np.arange(pos - n_keys + 1, pos + 1)
        want_att = go.sdpa(q_o, kc[ps % cap], vc[ps % cap], pos, pos - n_keys + 1, 0).reshape(-1)
        got_att = host(ops.sdpa_decode(dev(q_o.reshape(nh, hd)), dev(kc), dev(vc), pos, n_keys,
                                       ops.DecodeScratch(nh, nkv, hd, n_keys))).reshape(-1)
        close(got_att, want_att, 2e-3)
        ow, os_, ob = W(a + "o_proj.weight"), W(a + "o_proj.scales"), W(a + "o_proj.biases")
        want_o = go.qmm(want_att.reshape(1, -1), ow, os_, ob).reshape(-1)
        close(host(ops.quantized_matmul(dev(want_att.reshape(1, -1)), dev(ow), dev(os_), dev(ob))).reshape(-1), want_o)
        g3 = [W(p + "mlp.gate_proj" + s) for s in (".weight", ".scales", ".biases")]
        u3 = [W(p + "mlp.up_proj" + s) for s in (".weight", ".scales", ".biases")]

        def inter(g, u):
            r = g.shape[1]
            out = np.empty((2 * I, r), g.dtype)
            out.reshape(I // 16, 2, 16, r)[:, 0] = g.reshape(I // 16, 16, r)
            out.reshape(I // 16, 2, 16, r)[:, 1] = u.reshape(I // 16, 16, r)
            return out
        h1 = go.bf(go.fl(h) + go.fl(go.rms_norm(want_o.reshape(1, H), W(p + "post_attention_layernorm.weight"),
                                                  eps)).reshape(-1))
        xin = go.rms_norm(h1.reshape(1, H), W(p + "pre_feedforward_layernorm.weight"), eps)
        want_act = go.bf(go.fl(go.gelu_tanh(go.qmm(xin, *g3))) * go.fl(go.qmm(xin, *u3))).reshape(-1)
        hout = torch.zeros(H, dtype=torch.bfloat16, device="cuda")
        got_act = host(ops.qmv_fused(dev(want_o), *(dev(inter(g, u)) for g, u in zip(g3, u3)), prologue=2,
                                     epilogue=1, norm_w=dev(W(p + "pre_feedforward_layernorm.weight")),
                                     resid=dev(h), post_w=dev(W(p + "post_attention_layernorm.weight")), h_out=hout))
        assert np.array_equal(host(hout), h1)
        close(got_act, want_act)
        d3 = [W(p + "mlp.down_proj" + s) for s in (".weight", ".scales", ".biases")]
        want_dn = go.qmm(want_act.reshape(1, -1), *d3).reshape(-1)
        close(host(ops.quantized_matmul(dev(want_act.reshape(1, -1)), *(dev(x) for x in d3))).reshape(-1), want_dn)
        h2 = go.bf(go.fl(h1) + go.fl(go.rms_norm(want_dn.reshape(1, H), W(p + "post_feedforward_layernorm.weight"),
                                                   eps)).reshape(-1))
        h = go.bf(go.fl(h2) * go.fl(W(p + "layer_scalar"))[0])


@pytest.mark.parametrize("name,geo,seed,plen,steps", [
    ("cfg0", config0(), 7, 32, 64),
    ("tiny", tiny_fixture_geometry(), 11, 20, 24),
])
def test_greedy_matches_oracle(built_lib, oracle_lib, tmp_path, name, geo, seed, plen, steps):
    """Default (MLX CPU-stream) semantics: bf16-rounded attention scores amplify
    one-ulp differences in cached K (a score near a bf16 rounding boundary moves by
    a whole ulp, e.g. 0.125 at |s| ~ 20), so logits are compared loosely and the
    greedy tokens (teacher-forced, >= 99%) carry the parity claim."""
    eng, orc = _setup(tmp_path, geo, seed)
    agree, rels = _teacher_forced(eng, orc, _prompt(geo, plen, seed), steps)
    assert rels.max() <= 5e-2, rels
    assert agree.mean() >= 0.99, (agree, rels)


def test_free_running_greedy_cfg0(built_lib, oracle_lib, tmp_path):
    """Both sides run their own greedy loop (no teacher forcing)."""
    geo = config0()
    eng, orc = _setup(tmp_path, geo, 3)
    prompt = _prompt(geo, 32, 3)
    kv = eng.new_kv()
    f, _ = kv.prefill(prompt)
    toks = [f.token_id]
    for _ in range(64):
        f, _ = kv.decode(1)
        toks.append(f.token_id)
    okv = orc.new_kv()
    t0 = orc.prefill(okv, prompt)[0]
    otoks = [t0] + [o[0] for o in orc.decode(okv, 64)]
    agree = np.mean(np.asarray(toks) == np.asarray(otoks))
    assert agree >= 0.99, (toks, otoks)


def test_kv_cache_bytes_match_oracle_ring(built_lib, oracle_lib, tmp_path):
    """Ring slots (pos % (window + 8)) and global 256-step growth hold the same bf16 K/V."""
    geo = tiny_fixture_geometry()  # window 8: the ring wraps during the prompt
    eng, orc = _setup(tmp_path, geo, 5)
    prompt = _prompt(geo, 30, 5)
    kv = eng.new_kv()
    f, _ = kv.prefill(prompt)
    toks = [f.token_id]
    for _ in range(5):
        f, _ = kv.decode(1)
        toks.append(f.token_id)
    okv = orc.new_kv()
    orc.prefill(okv, prompt)
    orc.decode(okv, 5, forced=toks[:5])
    li = gi = 0
    for layer, kind in enumerate(geo.layer_types):
        for which in (0, 1):
            got = kv.copy_layer(layer, which)
            if kind == 0:
                ring = okv["local"][li]
                want = ring.k if which == 0 else ring.v
            else:
                gc = okv["global"][gi]
                want = gc.k if which == 0 else gc.v
            assert got.shape == want.shape, (layer, got.shape, want.shape)
            if layer == 0:
                # layer 0's K/V do not pass through attention: slot placement and values exact
                assert max_ulp(got, want) <= 1
                assert (got == want).mean() >= 0.99
            else:
                # deeper layers inherit the bf16-score amplification of earlier attention
                assert rel_l2(got, want) <= 5e-2
        if kind == 0:
            li += 1
        else:
            gi += 1


def test_chunked_prefill_matches_oracle(built_lib, oracle_lib, tmp_path):
    """A prompt longer than the 2048-token chunk exercises the continuation path."""
    geo = Geometry(hidden_size=256, intermediate_size=512, num_hidden_layers=3, layer_types=[0, 0, 1],
                   num_attention_heads=4, head_dim_local=64, head_dim_global=128, num_kv_heads_local=2,
                   num_kv_heads_global=1, sliding_window=128, vocab_size=512, max_position_embeddings=8192)
    eng, orc = _setup(tmp_path, geo, 21)
    prompt = _prompt(geo, 2300, 21)
    agree, rels = _teacher_forced(eng, orc, prompt, 4)
    assert rels.max() <= 5e-2, rels
    assert agree.all(), (agree, rels)


def test_abi_step_semantics_on_gpu(built_lib, tmp_path):
    geo = config0()
    d = tmp_path / "c"
    write_checkpoint(geo, str(d), seed=1)
    eng = hb.Engine(geo, weights_dir=str(d))
    L = built_lib
    kv = eng.new_kv()
    # decode before prefill
    assert L.hyp_decode_block(eng.handle, kv.handle, 1, eng._result) == hb.INVALID_ARGUMENT
    f, _ = kv.prefill(list(range(10)))
    # telemetry: ring = (128 + 8) slots * 2 heads * 64 * 2 bytes * (K and V); global = 256-step capacity
    assert f.local_kv_bytes == 136 * 2 * 64 * 2 * 2
    assert f.global_kv_bytes == 256 * 2 * 64 * 2 * 2
    # prefill again on a populated state
    arr = (ctypes.c_uint32 * 3)(1, 2, 3)
    ts = hb.HypTokenStream(ctypes.cast(arr, ctypes.POINTER(ctypes.c_uint32)), 3, 1)
    assert L.hyp_prefill_chunk(eng.handle, kv.handle, ctypes.byref(ts), eng._result) == hb.INVALID_ARGUMENT
    # zero-token decode is a no-op
    hb.check(L.hyp_decode_block(eng.handle, kv.handle, 0, eng._result))
    assert kv.cursor()[0] == 10
    # greedy through the sampled entry point with NULL config is identical
    kv2 = eng.new_kv()
    a, _ = kv2.prefill(list(range(10)))
    assert a.token_id == f.token_id and a.logit == f.logit
    # sampling config validation
    bad = hb.HypSamplingConfig(-1.0, 0, 0.0, 0.0, 1)
    assert L.hyp_decode_block_sampled(eng.handle, kv.handle, 1, ctypes.byref(bad), eng._result) == hb.INVALID_ARGUMENT
    bad = hb.HypSamplingConfig(1.0, 0, 0.0, 1.0, 1)
    assert L.hyp_decode_block_sampled(eng.handle, kv.handle, 1, ctypes.byref(bad), eng._result) == hb.INVALID_ARGUMENT
    # seeded sampling is reproducible
    cfg = hb.HypSamplingConfig(0.8, 40, 0.95, 0.0, 1234)
    kv3, kv4 = eng.new_kv(), eng.new_kv()
    kv3.prefill(list(range(10)))
    kv4.prefill(list(range(10)))
    s3, _ = kv3.decode(6, sampling=cfg)
    s4, _ = kv4.decode(6, sampling=cfg)
    assert s3.token_id == s4.token_id and s3.top_k_logprob_count == 8
    assert list(s3.top_k_logprob_values) == sorted(s3.top_k_logprob_values, reverse=True)
    # host-side fault after the first forward poisons the state (no device fault)
    hb.check(L.hyb_test_arm_post_append_fault())
    assert L.hyp_decode_block(eng.handle, kv.handle, 1, eng._result) == hb.INTERNAL
    assert "injected" in hb.last_error()
    assert L.hyp_decode_block(eng.handle, kv.handle, 1, eng._result) == hb.INTERNAL
    assert "free and recreate" in hb.last_error()
    # the poisoned state can still be freed; other states are unaffected
    kv.close()
    f5, _ = kv2.decode(1)
    assert f5.token_id < geo.vocab_size


def test_load_errors(built_lib, tmp_path):
    geo = config0()
    with pytest.raises(hb.HypError) as e:
        hb.Engine(geo, weights_dir=str(tmp_path / "missing"))
    assert e.value.status == hb.NOT_FOUND
    d = tmp_path / "empty"
    d.mkdir()
    with pytest.raises(hb.HypError) as e:
        hb.Engine(geo, weights_dir=str(d))
    assert e.value.status == hb.INTERNAL and "no .safetensors" in e.value.message
    # weight schema disagreeing with geometry (layer 1 declared sliding but has no v_proj)
    d2 = tmp_path / "c"
    write_checkpoint(geo, str(d2), seed=1)
    import dataclasses
    bad = dataclasses.replace(geo, num_hidden_layers=2, layer_types=[1, 1])
    with pytest.raises(hb.HypError) as e:
        hb.Engine(bad, weights_dir=str(d2))
    assert "disagrees with geometry" in e.value.message
