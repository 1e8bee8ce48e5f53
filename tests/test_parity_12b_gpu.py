"""End-to-end greedy parity at the BASELINE model shapes, against the CPU oracle.

The engine loads its seeded synthetic model on the device (hyb_model_load_synthetic);
the oracle rebuilds exactly the same tensors on the CPU (oracle.gemma_oracle
.synthetic_tensors restates the device generator: SplitMix64 codes and a table of
normal quantiles), so both sides run the same 12B- or 27B-shaped model without a
multi-gigabyte checkpoint on disk.

* Config 3 at full depth (48 layers, 5:1 sliding/global, window 1024, hd 256, 16/8
  heads, vocab 262144): a 64-token prompt through hyp_prefill_chunk, then 256 greedy
  hyp_decode_block steps. The oracle is teacher-forced with the engine's tokens, so
  every step compares the same input. This is the shape of the reference's own decode
  gate (native/hyperion_mlx/tests/forward_12b_decode_test.cc:5-18: greedy tokens exact
  over the decode, logits reported), with the north-star bar of >= 99% agreement.
* Config 4 (27B-shaped, 4 layers here to bound the oracle's CPU time): eight sequences
  with different prompt lengths stepped together through hyb_decode_batch, each
  compared with the oracle decoding that sequence alone.

Random-init weights give flat logit distributions (about 12% of steps have the top two
of 262144 logits within one bf16 ulp of each other), so a last-place rounding
difference anywhere in the 48 layers can swap a near-tied winner. The test reports the
agreement on every step and on the decisive steps (the oracle's winner ahead by more
than two bf16 ulps at its magnitude) and asserts >= 99% on both.
"""
import math

import numpy as np
import pytest

import hyperion_b200 as hb
from hyperion_b200.synth import bf16_bits_to_f32, config3, config4
from tests.conftest import has_gpu
from tests.gpu_util import rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_gpu(), reason="no CUDA device")]


def _ulp(v: float) -> float:
    """One bf16 unit in the last place at |v|."""
    if v == 0:
        return 2.0 ** -133
    return 2.0 ** (math.floor(math.log2(abs(v))) - 7)


def _gap_ulps(logits_bits: np.ndarray) -> float:
    """The oracle's winner lead over its runner-up, in bf16 ulps of the winner."""
    v = bf16_bits_to_f32(logits_bits).astype(np.float64)
    top2 = np.partition(v, -2)[-2:]
    return float((top2[1] - top2[0]) / _ulp(top2[1]))


def _oracle(geo, seed):
    from oracle import gemma_oracle as go
    return go.OracleModel(geo, go.synthetic_tensors(geo, seed), nthreads=go.host_threads())


def test_cfg3_48_layers_256_greedy_steps_match_oracle(built_lib, oracle_lib):
    geo = config3()
    seed = 31
    eng = hb.Engine(geo, synthetic_seed=seed)
    orc = _oracle(geo, seed)
    prompt = np.random.default_rng(seed).integers(0, geo.vocab_size, 64).tolist()
    kv = eng.new_kv()
    f, lg = kv.prefill(prompt, logits=True)
    okv = orc.new_kv()
    otok, _, _, olg = orc.prefill(okv, prompt)
    agree, rels, gaps = [f.token_id == otok], [rel_l2(lg, olg)], [_gap_ulps(olg)]
    prev = f.token_id
    for _ in range(256):
        f, lg = kv.decode(1, logits=True)
        (o_tok, _, _, o_lg), = orc.decode(okv, 1, forced=[prev])
        agree.append(f.token_id == o_tok)
        rels.append(rel_l2(lg, o_lg))
        gaps.append(_gap_ulps(o_lg))
        prev = f.token_id
    agree, rels, gaps = np.asarray(agree), np.asarray(rels), np.asarray(gaps)
    decisive = gaps > 2.0
    print(f"\ncfg3 48 layers: agreement {agree.mean():.4f} over {agree.size} samples "
          f"({(~agree).sum()} differ), decisive steps {decisive.sum()} agreement {agree[decisive].mean():.4f}; "
          f"logit rel-L2 median {np.median(rels):.2e} max {rels.max():.2e}; "
          f"differing steps' oracle gaps (ulps) {gaps[~agree].round(2).tolist()}")
    assert kv.cursor()[0] == len(prompt) + 256
    assert agree[decisive].mean() >= 0.99
    assert agree.mean() >= 0.99
    assert np.median(rels) <= 2e-2 and rels.max() <= 5e-2


def test_cfg4_batch8_matches_oracle(built_lib, oracle_lib):
    geo = config4(4)
    seed = 17
    eng = hb.Engine(geo, synthetic_seed=seed)
    orc = _oracle(geo, seed)
    rng = np.random.default_rng(seed)
    lens = [9, 40, 17, 64, 23, 5, 33, 48]
    prompts = [rng.integers(0, geo.vocab_size, n).tolist() for n in lens]
    kvs, okvs, inputs, agree, dlog = [], [], [], [], []
    for p in prompts:
        kv = eng.new_kv()
        f, _ = kv.prefill(p)
        okv = orc.new_kv()
        otok, ologit, _, _ = orc.prefill(okv, p)
        agree.append(f.token_id == otok)
        kvs.append(kv)
        okvs.append(okv)
        inputs.append(f.token_id)
    for _ in range(4):
        toks, logs = eng.decode_batch(kvs)
        for i, okv in enumerate(okvs):
            (o_tok, o_logit, _, _), = orc.decode(okv, 1, forced=[inputs[i]])
            agree.append(toks[i] == o_tok)
            if toks[i] == o_tok:
                dlog.append(abs(logs[i] - o_logit) / max(1.0, abs(o_logit)))
        inputs = toks
    agree = np.asarray(agree)
    print(f"\ncfg4 batch 8: agreement {agree.mean():.4f} over {agree.size}, top-logit rel diff max {max(dlog):.2e}")
    assert agree.mean() >= 0.99, agree
    assert max(dlog) <= 2 ** -5
