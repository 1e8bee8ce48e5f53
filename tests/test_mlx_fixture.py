"""The reference's MLX-written tiny checkpoint (tests/golden/gemma4_unified_tiny).

The reference generated it with MLX itself (mx.quantize g64/b4 affine and
mx.save_safetensors, crates/hyperion-model/fixtures/build_gemma4_unified_tiny.py:53-57,
129-130); tests/golden/copy_mlx_fixture.py copied it byte for byte. The CPU tests here
pin the copy (SHA-256), its geometry against the engine's tiny geometry, and the tensor
schema the reference loader requires (weights_loader.cc:72-154: mlx-lm names, U32 codes
and BF16 scales/biases per quantized linear, no v_proj on the global layer). The GPU
test (bottom) loads the same directory through hyp_model_load and decodes it beside the
oracle running on the same tensors.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from hyperion_b200.safetensors_io import read_checkpoint_dir
from hyperion_b200.synth import tiny_fixture_geometry
from tests.conftest import has_gpu

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "gemma4_unified_tiny")
PROMPT = [7, 3, 40, 100, 5, 77, 12, 64, 90, 2, 31, 8]  # starts with forward_test.cc's {7, 3, 40, 100}


def test_fixture_copy_is_intact():
    with open(os.path.join(FIXTURE, "SHA256SUMS")) as f:
        for line in f:
            digest, name = line.split()
            with open(os.path.join(FIXTURE, name), "rb") as fh:
                assert hashlib.sha256(fh.read()).hexdigest() == digest, name


def test_fixture_geometry_matches_tiny_geometry():
    with open(os.path.join(FIXTURE, "config.json")) as f:
        tc = json.load(f)["text_config"]
    g = tiny_fixture_geometry()
    assert tc["hidden_size"] == g.hidden_size and tc["intermediate_size"] == g.intermediate_size
    assert tc["num_hidden_layers"] == g.num_hidden_layers
    assert [1 if k == "full_attention" else 0 for k in tc["layer_types"]] == g.layer_types
    assert tc["num_attention_heads"] == g.num_attention_heads
    assert tc["head_dim"] == g.head_dim_local and tc["global_head_dim"] == g.head_dim_global
    assert tc["num_key_value_heads"] == g.num_kv_heads_local
    assert tc["num_global_key_value_heads"] == g.num_kv_heads_global
    assert tc["sliding_window"] == g.sliding_window and tc["vocab_size"] == g.vocab_size
    assert tc["attention_k_eq_v"] and tc["final_logit_softcapping"] == g.final_logit_softcapping
    rp = tc["rope_parameters"]
    assert rp["sliding_attention"]["rope_theta"] == g.rope_theta_local
    assert rp["full_attention"]["rope_theta"] == g.rope_theta_global
    assert rp["full_attention"]["partial_rotary_factor"] == g.partial_rotary_factor_global


def test_fixture_schema():
    t = read_checkpoint_dir(FIXTURE)
    g = tiny_fixture_geometry()
    H = g.hidden_size
    pre = "language_model.model."
    assert t[pre + "embed_tokens.weight"].dtype == np.uint32
    assert t[pre + "embed_tokens.weight"].shape == (g.vocab_size, H // 8)
    assert t[pre + "embed_tokens.scales"].shape == (g.vocab_size, H // 64)
    for i, kind in enumerate(g.layer_types):
        a = f"{pre}layers.{i}.self_attn."
        hd, nkv = g.head_dim(i), g.n_kv(i)
        assert t[a + "q_proj.weight"].shape == (g.num_attention_heads * hd, H // 8)
        assert t[a + "k_proj.weight"].shape == (nkv * hd, H // 8)
        assert (a + "v_proj.weight" in t) == (kind == 0)  # the global layer derives V from K
        assert t[a + "q_proj.scales"].dtype == np.uint16 and t[a + "q_proj.biases"].dtype == np.uint16
        assert t[f"{pre}layers.{i}.mlp.down_proj.weight"].shape == (H, g.intermediate_size // 8)


def test_oracle_decodes_fixture(oracle_lib):
    from oracle import gemma_oracle as go
    geo = tiny_fixture_geometry()
    orc = go.OracleModel(geo, read_checkpoint_dir(FIXTURE))
    kv = orc.new_kv()
    tok = orc.prefill(kv, PROMPT)[0]
    toks = [o[0] for o in orc.decode(kv, 8)]
    assert 0 <= tok < geo.vocab_size and all(0 <= t < geo.vocab_size for t in toks)
    assert kv["offset"] == len(PROMPT) + 8


@pytest.mark.gpu
@pytest.mark.skipif(not has_gpu(), reason="no CUDA device")
def test_engine_loads_mlx_checkpoint_and_matches_oracle(built_lib, oracle_lib):
    """hyp_model_load on the MLX-written directory (two shards plus the index file, the
    tied embedding, K = V on the global layer, norm weights used as stored), then a
    prefill and 24 greedy decode steps teacher-forced against the oracle on the same
    tensors; the ring (window 8, capacity 16) wraps during the run."""
    import hyperion_b200 as hb
    from oracle import gemma_oracle as go
    from tests.gpu_util import max_ulp, rel_l2
    geo = tiny_fixture_geometry()
    t = read_checkpoint_dir(FIXTURE)
    eng = hb.Engine(geo, weights_dir=FIXTURE)
    orc = go.OracleModel(geo, t)
    kv = eng.new_kv()
    f, lg = kv.prefill(PROMPT, logits=True)
    okv = orc.new_kv()
    otok, _, _, olg = orc.prefill(okv, PROMPT)
    agree, rels = [f.token_id == otok], [rel_l2(lg, olg)]
    prev = f.token_id
    for _ in range(24):
        f, lg = kv.decode(1, logits=True)
        (o_tok, _, _, o_lg), = orc.decode(okv, 1, forced=[prev])
        agree.append(f.token_id == o_tok)
        rels.append(rel_l2(lg, o_lg))
        prev = f.token_id
    print(f"\nMLX fixture: agreement {np.mean(agree):.3f}, logit rel-L2 max {max(rels):.2e}")
    assert np.mean(agree) >= 0.99, agree
    assert max(rels) <= 5e-2, rels
    # layer 0's cache rows never pass through attention: placement and values exact
    ring = okv["local"][0]
    for which, want in ((0, ring.k), (1, ring.v)):
        got = kv.copy_layer(0, which)
        assert got.shape == want.shape
        assert max_ulp(got, want) <= 1 and (got == want).mean() >= 0.99
