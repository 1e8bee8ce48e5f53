"""The sampler's random draw and the oracle's sampler on the CPU.

The reference draws each sampled token from std::uniform_real_distribution<float>(0, sz)
over a freshly seeded std::mt19937_64 (native/hyperion_mlx/src/forward.cc:290-295). The
device sampler (hyperion_b200/csrc/sampler.cu) computes that draw itself from the
published MT19937-64 algorithm: the first output needs words 0, 1 and 156 of the seeding,
one twist and the tempering, and the float conversion of generate_canonical. This file
restates those steps in Python and pins them against the toolchain's own standard library
(oracle/std_rng.cc), so the constants the device uses are the standard's.
"""
import numpy as np
import pytest

M64 = (1 << 64) - 1


def mt64_first(seed: int) -> int:
    x = seed & M64
    w = [x]
    for i in range(1, 157):
        x = (6364136223846793005 * (x ^ (x >> 62)) + i) & M64
        w.append(x)
    y = (w[0] & 0xFFFFFFFF80000000) | (w[1] & 0x7FFFFFFF)
    z = w[156] ^ (y >> 1) ^ (0xB5026F5AA96619E9 if y & 1 else 0)
    z ^= (z >> 29) & 0x5555555555555555
    z ^= (z << 17) & 0x71D67FFFEDA60000 & M64
    z ^= (z << 37) & 0xFFF7EEE000000000 & M64
    z ^= z >> 43
    return z & M64


def uniform_draw(seed: int, b: float) -> np.float32:
    r = np.float32(float(mt64_first(seed))) * np.float32(2.0 ** -64)
    if r >= 1.0:
        r = np.nextafter(np.float32(1.0), np.float32(0.0))
    return np.float32(r * np.float32(b))


SEEDS = [0, 1, 2, 42, 1234, 5489, 2 ** 32 + 7, 2 ** 63 - 1, 2 ** 64 - 1, 0xDEADBEEFCAFEF00D] + \
    [int(s) for s in np.random.default_rng(3).integers(0, 2 ** 63, 200)]


def test_mt19937_64_first_output_matches_the_standard_library(oracle_lib):
    from oracle import gemma_oracle as go
    L = go.rng_lib()
    for s in SEEDS:
        assert mt64_first(s) == L.orc_mt19937_64_first(s), s


def test_uniform_float_draw_matches_the_standard_library(oracle_lib):
    from oracle import gemma_oracle as go
    L = go.rng_lib()
    for s in SEEDS:
        for b in (1.0, 3.5, 123.25, 1e-3):
            assert uniform_draw(s, b) == np.float32(L.orc_uniform_float_draw(s, b)), (s, b)


def _row(n, seed):
    from hyperion_b200.synth import f32_to_bf16_bits
    x = np.random.default_rng(seed).standard_normal(n).astype(np.float32) * 2.0
    return f32_to_bf16_bits(30.0 * np.tanh(x / 30.0))


def test_oracle_sampler_filters(oracle_lib):
    """Greedy limits and filter counts of the oracle sampler on a small row."""
    from oracle import gemma_oracle as go
    row = _row(4096, 1)
    vals = go.fl(row)
    tok, logit, u, sz, kept, top, topv = go.sample(row, 1.0, top_k=1, seed=9)
    assert kept == 1 and tok == int(np.argmax(vals)) and logit == vals.max()
    _, _, _, _, kept, _, _ = go.sample(row, 1.0, top_k=40, seed=9)
    assert kept == 40
    _, _, _, _, kept_all, _, _ = go.sample(row, 1.0, seed=9)
    assert kept_all == 4096
    _, _, _, _, kept_p, _, _ = go.sample(row, 0.5, top_p=0.5, seed=9)
    assert 1 <= kept_p < 4096
    assert list(topv) == sorted(topv, reverse=True) and len(top) == 8
    # the same seed draws the same token
    assert go.sample(row, 0.8, top_k=50, top_p=0.9, seed=77)[0] == go.sample(row, 0.8, top_k=50, top_p=0.9, seed=77)[0]
