"""Greedy speculative verify (hyb_verify) against plain decode on the same states.

One verify pass runs [last token, draft...] through the chunked forward at consecutive
positions and samples every row; plain decode reaches the same rows one step at a time.
The comparison is teacher-forced: a clone taken before the pass is stepped through the
same inputs with hyb_decode_forced, so every row of the pass has a decode twin. The
forward GEMM rounds its bf16 products in a different order from the decode qmv, so the
logits may differ in the last bf16 places; greedy tokens must agree >= 99% and the top
logits within 2**-5 relative. After a partial acceptance the rejected tail sits in the
ring's speculative slack (capacity window + 8); decoding on from the committed cursor must
match a twin that never saw the tail, which the tiny geometry (window 8, ring 16) checks
with the ring wrapping on every pass.
"""
import numpy as np
import pytest

import hyperion_b200 as hb
from hyperion_b200.synth import config0, config3, config4, tiny_fixture_geometry
from tests.conftest import has_gpu
from tests.gpu_util import rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not has_gpu(), reason="no CUDA device")]

LOGIT_TOL = 2.0 ** -5


def _forced_twin(kv, inputs):
    """Greedy samples of a clone of `kv` teacher-forced through `inputs`."""
    tw = kv.clone()
    out = []
    for t in inputs:
        f, _ = tw.decode(1, forced=t)
        out.append((f.token_id, f.logit))
    tw.close()
    return out


def _draft(rng, truth, vocab, n):
    """A draft that follows `truth` for a random number of tokens, then guesses."""
    keep = int(rng.integers(0, n + 1))
    d = list(truth[:keep]) + rng.integers(0, vocab, n - keep).tolist()
    return d[:n]


def _run(geo, seed, prompt_len, passes, n_max):
    eng = hb.Engine(geo, synthetic_seed=seed)
    rng = np.random.default_rng(seed)
    kv = eng.new_kv()
    kv.prefill(rng.integers(0, geo.vocab_size, prompt_len).tolist())
    agree, dlog, accepted = [], [], []
    for _ in range(passes):
        n = int(rng.integers(1, n_max + 1))
        off, last = kv.cursor()
        # the model's own continuation, so acceptance varies between 0 and n
        truth = [t for t, _ in _forced_twin(kv, [last])]
        tw = kv.clone()
        for _ in range(n - 1):
            f, _ = tw.decode(1)
            truth.append(f.token_id)
        tw.close()
        draft = _draft(rng, truth, geo.vocab_size, n)
        ref = _forced_twin(kv, [last] + draft)
        a, toks, logs = kv.verify(draft)
        for i in range(n + 1):
            agree.append(toks[i] == ref[i][0])
            if toks[i] == ref[i][0]:
                dlog.append(abs(logs[i] - ref[i][1]) / max(1.0, abs(ref[i][1])))
        exp_a = 0
        while exp_a < n and draft[exp_a] == toks[exp_a]:
            exp_a += 1
        assert a == exp_a
        assert kv.cursor() == (off + a + 1, toks[a])
        accepted.append(a)
    return np.asarray(agree), np.asarray(dlog), accepted


@pytest.mark.parametrize("name,geo,prompt_len,passes", [
    ("tiny_ring_wraps", tiny_fixture_geometry(), 21, 24),
    ("cfg0", config0(), 150, 16),
    ("cfg3_4layers", config3(4), 1030, 6),
    ("cfg4_3layers", config4(3), 300, 6),
])
def test_verify_matches_decode(built_lib, name, geo, prompt_len, passes):
    agree, dlog, accepted = _run(geo, 31, prompt_len, passes, 8)
    assert agree.mean() >= 0.99, agree
    assert dlog.max() <= LOGIT_TOL, dlog.max()
    assert max(accepted) > 0  # some drafts were (partly) right


def test_verify_rejected_tail_is_invisible(built_lib):
    """After passes with rejected tails, decoding on matches a twin that took only the
    accepted tokens by plain decode: the tail in the ring slack never reaches the window
    (tiny geometry: window 8, ring 16, so every 9-row pass wraps the ring)."""
    geo = tiny_fixture_geometry()
    eng = hb.Engine(geo, synthetic_seed=9)
    rng = np.random.default_rng(9)
    a_kv = eng.new_kv()
    a_kv.prefill(rng.integers(0, geo.vocab_size, 13).tolist())
    b_kv = a_kv.clone()
    total_tail = 0
    for _ in range(10):
        _, last = a_kv.cursor()
        probe = a_kv.clone()
        f, _ = probe.decode(1)  # the first draft token is the model's own
        probe.close()
        draft = [f.token_id] + [(f.token_id + 1 + i) % geo.vocab_size for i in range(7)]
        a, _, _ = a_kv.verify(draft)
        total_tail += 8 - a
        for t in [last] + draft[:a]:  # the twin: a + 1 plain steps through the same inputs
            b_kv.decode(1, forced=t)
        assert a_kv.cursor()[0] == b_kv.cursor()[0]
    assert total_tail > 0
    agree = []
    for _ in range(12):
        _, t = b_kv.cursor()
        fa, la = a_kv.decode(1, logits=True, forced=t)
        fb, lb = b_kv.decode(1, logits=True, forced=t)
        agree.append(fa.token_id == fb.token_id)
        assert rel_l2(np.asarray(la), np.asarray(lb)) <= 1e-2
    assert np.mean(agree) >= 11 / 12


@pytest.mark.parametrize("name,geo,seed,plen,passes", [
    ("cfg0", config0(), 7, 32, 10),
    ("tiny_ring_wraps", tiny_fixture_geometry(), 11, 20, 12),
])
def test_verify_matches_oracle(built_lib, oracle_lib, tmp_path, name, geo, seed, plen, passes):
    """Every row of every verify pass against the CPU oracle teacher-forced through the
    same inputs from its own committed state (a copy per pass); the oracle then commits
    the same accepted rows. Drafts follow the oracle's own greedy continuation up to a
    random point, so acceptance varies. Greedy tokens >= 99%; post-softcap top logits
    within 5e-2 relative (the bound of the decode-vs-oracle tests)."""
    import copy
    from oracle import gemma_oracle as go
    from hyperion_b200.synth import bf16_bits_to_f32, write_checkpoint
    t = write_checkpoint(geo, str(tmp_path / "w"), seed=seed)
    eng, orc = hb.Engine(geo, weights_dir=str(tmp_path / "w")), go.OracleModel(geo, t)
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, geo.vocab_size, plen).tolist()
    kv, okv = eng.new_kv(), orc.new_kv()
    kv.prefill(prompt)
    orc.prefill(okv, prompt)
    agree, rel, accepted = [], [], []
    for _ in range(passes):
        n = int(rng.integers(1, 9))
        _, last = kv.cursor()
        probe = copy.deepcopy(okv)
        seq, inp = [], last
        for _ in range(n):  # the oracle's own greedy continuation from `last`
            (tok, _, _, _), = orc.decode(probe, 1, forced=[inp])
            seq.append(tok)
            inp = tok
        keep = int(rng.integers(0, n + 1))
        draft = seq[:keep] + rng.integers(0, geo.vocab_size, n - keep).tolist()
        a, toks, logs = kv.verify(draft)
        ref = orc.decode(copy.deepcopy(okv), n + 1, forced=[last] + draft)
        for i in range(n + 1):
            agree.append(toks[i] == ref[i][0])
            if toks[i] == ref[i][0]:
                want = float(bf16_bits_to_f32(np.asarray([ref[i][3][toks[i]]], dtype=np.uint16))[0])
                rel.append(abs(logs[i] - want) / max(1.0, abs(want)))
        orc.decode(okv, a + 1, forced=[last] + draft[:a])  # commit what the engine committed
        assert kv.cursor()[0] == okv["offset"]
        accepted.append(a)
    assert np.mean(agree) >= 0.99, agree
    assert max(rel) <= 5e-2, max(rel)
    assert max(accepted) > 0


def test_verify_errors(built_lib):
    geo = config0()
    eng = hb.Engine(geo, synthetic_seed=2)
    kv = eng.new_kv()
    with pytest.raises(hb.HypError) as e:
        kv.verify([1, 2])  # not populated
    assert e.value.status == hb.INVALID_ARGUMENT
    kv.prefill([5, 6, 7])
    for bad in ([], list(range(9)), [geo.vocab_size]):
        with pytest.raises(hb.HypError) as e:
            kv.verify(bad)
        assert e.value.status == hb.INVALID_ARGUMENT
    assert kv.cursor()[0] == 3  # rejected calls leave the state alone
    a, toks, _ = kv.verify([1])
    assert kv.cursor() == (4 + a, toks[a])
