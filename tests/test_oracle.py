"""CPU checks of the oracle itself: nibble order, exactness against an independent
numpy restatement, attention semantics, and the committed golden vectors."""
import os

import numpy as np
import pytest

from hyperion_b200.synth import (bf16_bits_to_f32, f32_to_bf16_bits, pack_q4, random_q4, affine_quantize,
                                 config0, make_weights)

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def unpack_np(w):
    n, k8 = w.shape
    q = np.zeros((n, k8 * 8), dtype=np.uint8)
    for i in range(8):
        q[:, i::8] = (w >> np.uint32(4 * i)) & 0xF
    return q


def test_pack_unpack_roundtrip_bit_exact(oracle_lib):
    from oracle import gemma_oracle as go
    rng = np.random.default_rng(1)
    q = rng.integers(0, 16, size=(7, 256), dtype=np.uint32)
    w = pack_q4(q)
    assert np.array_equal(unpack_np(w), q)
    out = np.empty(256, dtype=np.uint8)
    for n in range(7):
        go.lib().orc_unpack_row(w.ctypes.data, 256, n, out.ctypes.data)
        assert np.array_equal(out, q[n])
    # code 8j+i sits in bits [4i, 4i+4) of word j
    assert (int(w[0, 0]) & 0xF) == q[0, 0] and ((int(w[0, 0]) >> 28) & 0xF) == q[0, 7]


@pytest.mark.parametrize("M,K,N", [(1, 64, 8), (1, 256, 64), (3, 512, 40), (2, 1024, 17)])
def test_orc_qmm_matches_float64_dequant(oracle_lib, M, K, N):
    from oracle import gemma_oracle as go
    rng = np.random.default_rng(K + N)
    w, s, b = random_q4(rng, N, K)
    x = f32_to_bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    q = unpack_np(w).astype(np.float64)
    sf = bf16_bits_to_f32(s).astype(np.float64).repeat(64, axis=1)
    bfv = bf16_bits_to_f32(b).astype(np.float64).repeat(64, axis=1)
    what = sf * q + bfv
    ref = bf16_bits_to_f32(x).astype(np.float64) @ what.T
    y = go.qmm(x, w, s, b)
    assert np.array_equal(y, f32_to_bf16_bits(ref.astype(np.float32)))


def _sdpa_np(q, k, v, qp0, kp0, window, mode):
    Lq, H, D = q.shape
    Lk, Hkv, _ = k.shape
    rep = H // Hkv
    qf, kf, vf = (bf16_bits_to_f32(a).astype(np.float64) for a in (q, k, v))
    out = np.zeros((Lq, H, D))
    for i in range(Lq):
        for h in range(H):
            s = kf[:, h // rep, :] @ qf[i, h]
            if mode == 0:
                s = bf16_bits_to_f32(f32_to_bf16_bits(s.astype(np.float32))).astype(np.float64)
            kp = kp0 + np.arange(Lk)
            qp = qp0 + i
            vis = (kp <= qp) & ((window == 0) | (kp > qp - window))
            s = np.where(vis, s, -np.inf)
            p = np.exp(s - s.max())
            p /= p.sum()
            if mode == 0:
                p = bf16_bits_to_f32(f32_to_bf16_bits(p.astype(np.float32))).astype(np.float64)
            out[i, h] = p @ vf[:, h // rep, :]
    return f32_to_bf16_bits(out.astype(np.float32))


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("window", [0, 5])
def test_orc_sdpa_semantics(oracle_lib, mode, window):
    from oracle import gemma_oracle as go
    rng = np.random.default_rng(3)
    Lq, Lk, H, Hkv, D = 4, 11, 4, 2, 64
    q = f32_to_bf16_bits(rng.standard_normal((Lq, H, D), dtype=np.float32))
    k = f32_to_bf16_bits(rng.standard_normal((Lk, Hkv, D), dtype=np.float32) * 0.3)
    v = f32_to_bf16_bits(rng.standard_normal((Lk, Hkv, D), dtype=np.float32))
    got = go.sdpa(q, k, v, 7, 0, window, mode=mode)
    want = _sdpa_np(q, k, v, 7, 0, window, mode)
    diff = np.abs(bf16_bits_to_f32(got) - bf16_bits_to_f32(want))
    assert diff.max() <= 2 ** -7 * np.abs(bf16_bits_to_f32(want)).max()
    assert (got == want).mean() > 0.98


def test_gelu_constants_are_bf16():
    from oracle import gemma_oracle as go
    assert go._BF_C == 0.044677734375 and go._BF_K == 0.796875


def test_affine_quantize_roundtrip_error():
    rng = np.random.default_rng(5)
    wf = (rng.standard_normal((16, 128)) * 0.02).astype(np.float32)
    w, s, b = affine_quantize(wf)
    q = unpack_np(w).astype(np.float32)
    deq = bf16_bits_to_f32(s).repeat(64, 1) * q + bf16_bits_to_f32(b).repeat(64, 1)
    rng_w = np.ptp(wf.reshape(16, 2, 64), axis=-1).repeat(64, 1)
    # the edge-anchored scale can clip the far end of a group by up to one step;
    # plus the bf16 rounding of the stored scale and bias
    bound = np.abs(bf16_bits_to_f32(s)).repeat(64, 1) * 1.0 + 2 ** -7 * np.abs(wf).max() + 1e-6
    assert np.all(rng_w > 0)
    assert np.all(np.abs(deq - wf) <= bound)


@pytest.mark.skipif(not os.path.exists(os.path.join(GOLDEN, "oracle_golden.npz")), reason="golden not generated")
def test_oracle_reproduces_committed_golden(oracle_lib):
    """The oracle's outputs on seeded inputs are pinned by tests/golden (make_golden.py)."""
    from tests.golden.make_golden import compute
    g = np.load(os.path.join(GOLDEN, "oracle_golden.npz"))
    now = compute()
    for key in g.files:
        assert np.array_equal(g[key], now[key]), key
