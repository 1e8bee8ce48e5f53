// std_rng.cc - the C++ standard library's random draw the reference sampler makes.
//
// TEST INFRASTRUCTURE ONLY (see oracle/hyp_oracle.c). The reference draws each sampled
// token with std::uniform_real_distribution<float>(0, sz) over a freshly seeded
// std::mt19937_64 (native/hyperion_mlx/src/forward.cc:290-295). These wrappers expose that
// exact draw, from the toolchain's own standard library, to the oracle and its tests.
#include <cstdint>
#include <random>

extern "C" uint64_t orc_mt19937_64_first(uint64_t seed) {
    std::mt19937_64 g(seed);
    return g();
}

extern "C" float orc_uniform_float_draw(uint64_t seed, float b) {
    std::mt19937_64 g(seed);
    std::uniform_real_distribution<float> u(0.0f, b);
    return u(g);
}
