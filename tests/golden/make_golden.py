"""Generate tests/golden/oracle_golden.npz: the oracle's outputs on small seeded
inputs (quantized matmul, attention, and end-to-end greedy runs of config 0 and
of the reference tiny-fixture geometry with synthetic weights).

These pin the oracle against silent changes; they are regenerated only when the
oracle's semantics are deliberately changed.

Run: python -m tests.golden.make_golden
"""
import os

import numpy as np

from hyperion_b200.synth import config0, f32_to_bf16_bits, make_weights, random_q4, tiny_fixture_geometry

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "oracle_golden.npz")


def compute():
    from oracle import gemma_oracle as go
    rng = np.random.default_rng(20260101)
    out = {}
    w, s, b = random_q4(rng, 96, 512)
    x = f32_to_bf16_bits(rng.standard_normal((3, 512), dtype=np.float32))
    out["qmm_x"], out["qmm_w"], out["qmm_s"], out["qmm_b"] = x, w, s, b
    out["qmm_y"] = go.qmm(x, w, s, b)
    q = f32_to_bf16_bits(rng.standard_normal((5, 4, 64), dtype=np.float32))
    k = f32_to_bf16_bits(rng.standard_normal((9, 2, 64), dtype=np.float32) * 0.25)
    v = f32_to_bf16_bits(rng.standard_normal((9, 2, 64), dtype=np.float32))
    out["sdpa_q"], out["sdpa_k"], out["sdpa_v"] = q, k, v
    out["sdpa_out_w3"] = go.sdpa(q, k, v, 4, 0, 3)
    out["sdpa_out_full"] = go.sdpa(q, k, v, 4, 0, 0)
    for name, geo, seed, plen, steps in (("cfg0", config0(), 7, 32, 8),
                                         ("tiny", tiny_fixture_geometry(), 11, 20, 8)):
        m = go.OracleModel(geo, make_weights(geo, seed))
        kv = m.new_kv()
        prompt = np.random.default_rng(seed).integers(0, geo.vocab_size, plen).tolist()
        tok, logit, tie, lg = m.prefill(kv, prompt)
        toks = [tok] + [o[0] for o in m.decode(kv, steps)]
        out[f"{name}_tokens"] = np.asarray(toks, dtype=np.int64)
        out[f"{name}_prefill_logits"] = lg
    return out


if __name__ == "__main__":
    np.savez_compressed(OUT, **compute())
    print("wrote", OUT, os.path.getsize(OUT), "bytes")
