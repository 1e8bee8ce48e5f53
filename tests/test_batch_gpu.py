"""Batched decode (hyb_decode_batch) against one-sequence decode on the same states.

Every sequence of a batch is prefilled with its own prompt (different lengths, so the
batch mixes positions and KV lengths), then stepped together; a twin state of each
sequence is stepped alone through hyb_decode_forced with the same input tokens
(teacher forcing). The batched projections dequantise the codes to fp16 before the
tensor-core product while the batch-1 path folds scale and bias in fp32 after it, so
the logits may differ in the last bf16 place; greedy tokens must agree >= 99% and the
top logits within two bf16 ulps.
"""
import numpy as np
import pytest

import hyperion_b200 as hb
from hyperion_b200.synth import config0, config3, config4
from tests.conftest import has_gpu

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_gpu(), reason="no CUDA device")]


def _run(geo, seed, lens, steps):
    eng = hb.Engine(geo, synthetic_seed=seed)
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, geo.vocab_size, n).tolist() for n in lens]
    batch, twins, first = [], [], []
    for p in prompts:
        kb, kt = eng.new_kv(), eng.new_kv()
        fb, _ = kb.prefill(p)
        ft, _ = kt.prefill(p)
        assert fb.token_id == ft.token_id
        batch.append(kb)
        twins.append(kt)
        first.append(fb.token_id)
    inputs = list(first)
    agree, dlog = [], []
    for _ in range(steps):
        toks, logs = eng.decode_batch(batch)
        for i, kt in enumerate(twins):
            f, _ = kt.decode(1, forced=inputs[i])
            agree.append(toks[i] == f.token_id)
            if toks[i] == f.token_id:
                dlog.append(abs(logs[i] - f.logit) / max(1.0, abs(f.logit)))
        inputs = toks
    for kb, kt in zip(batch, twins):
        assert kb.cursor()[0] == kt.cursor()[0]
    return np.asarray(agree), np.asarray(dlog)


@pytest.mark.parametrize("name,geo,lens,steps", [
    ("cfg0_b3", config0(), [20, 33, 47], 16),
    ("cfg0_b10", config0(), [5 + 7 * i for i in range(10)], 8),
    ("cfg3_4layers_b5", config3(4), [40, 41, 130, 7, 64], 6),
    ("cfg4_3layers_b9", config4(3), [30, 64, 17, 90, 33, 12, 50, 71, 8], 4),
])
def test_decode_batch_matches_single(built_lib, name, geo, lens, steps):
    agree, dlog = _run(geo, 21, lens, steps)
    assert agree.mean() >= 0.99, agree
    assert dlog.max() <= 2 ** -6, dlog.max()


def test_decode_batch_above_qmv_reach_262k_vocab(built_lib):
    """20 sequences take the tcgen05 GEMM path, whose lm_head runs over the 262144-row
    vocabulary in slices unpacked in turn from the packed table (a ragged last slice)."""
    agree, dlog = _run(config3(2), 33, [9 + 5 * i for i in range(20)], 2)
    assert agree.mean() >= 0.97, agree
    assert dlog.max() <= 2 ** -6, dlog.max()


def test_decode_batch_64(built_lib):
    """The largest batch (8 MMA column groups), sequences at 64 different positions."""
    geo = config0()
    agree, dlog = _run(geo, 5, [3 + (i * 37) % 150 for i in range(64)], 3)
    assert agree.mean() >= 0.99
    assert dlog.max() <= 2 ** -6


def test_decode_batch_errors(built_lib):
    geo = config0()
    eng = hb.Engine(geo, synthetic_seed=1)
    a, b = eng.new_kv(), eng.new_kv()
    a.prefill([1, 2, 3])
    with pytest.raises(hb.HypError) as e:
        eng.decode_batch([a, b])  # b is not populated
    assert e.value.status == hb.INVALID_ARGUMENT
    with pytest.raises(hb.HypError) as e:
        eng.decode_batch([a, a])
    assert "twice" in e.value.message
    with pytest.raises(hb.HypError):
        eng.decode_batch([])
    toks, _ = eng.decode_batch([a])  # a batch of one is the plain step
    assert a.cursor() == (4, toks[0])


def test_kvstate_clone(built_lib):
    """A clone decodes exactly like its source; its own last token redirects it."""
    geo = config0()
    eng = hb.Engine(geo, synthetic_seed=3)
    a = eng.new_kv()
    f, _ = a.prefill(list(range(40)))
    b = a.clone()
    c = a.clone(last_token=7)
    assert b.cursor() == a.cursor() and c.cursor() == (a.cursor()[0], 7)
    for _ in range(5):
        fa, la = a.decode(1, logits=True)
        fb, lb = b.decode(1, logits=True)
        assert fa.token_id == fb.token_id and np.array_equal(np.asarray(la), np.asarray(lb))
    toks, _ = eng.decode_batch([c, a.clone(last_token=9), a.clone(last_token=9)])
    assert toks[1] == toks[2]
