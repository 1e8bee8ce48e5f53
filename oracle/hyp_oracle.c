/*
 * hyp_oracle.c - CPU restatement of the Hyperion decode/prefill arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * engine and the timed host-CPU baseline; nothing in the product path
 * (hyperion_b200/) links or calls it. Only tests/, __graft_entry__.smoke()
 * and bench.py (its cpu_baseline / --impl reference legs) may load it.
 *
 * What it restates (reference paths are inside jscott3201/hyperion):
 *   - orc_qmm: QuantizedLinear::apply -> mx::quantized_matmul(x, w, scales,
 *     biases, transpose=true, group_size=64, bits=4, "affine")
 *     (native/hyperion_mlx/src/weights.h:26-37). MLX's published affine
 *     definition: w_hat[n,k] = scales[n,k/64] * q[n,k] + biases[n,k/64], with
 *     q[n, 8j+i] stored in bits [4i, 4i+4) of word j of row n. The sum is
 *     evaluated as sum_g s*sum(q*x) + b*sum(x): each group dot is exact in
 *     float (integer q times bf16 x, 64 terms) and groups are combined in
 *     double, so the result is the correctly rounded bf16 of the exact value
 *     up to double rounding.
 *   - orc_sdpa: mx::fast::scaled_dot_product_attention with a boolean mask as
 *     it evaluates on MLX's CPU stream (forward.cc:498-504): scores are a bf16
 *     matmul (fp32 accumulate, bf16 result), masked positions take bf16's
 *     lowest value, softmax is "precise" (fp32 math, bf16 result), and the
 *     probability-times-V matmul accumulates in fp32 and returns bf16. GQA maps
 *     query head h to KV head h / (H / Hkv). mode=1 skips the two bf16
 *     roundings (fused-kernel semantics) for comparison.
 *
 * Threading: OpenMP over output rows; `nthreads` <= 0 uses the OpenMP default.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Round-to-nearest-even float -> bf16 (NaN kept quiet). */
static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static inline uint16_t d2bf(double d) { return f2bf((float)d); }

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

int orc_version(void) { return 1; }

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Unpack row n's K codes (bit-exact nibble order) into out[K]. */
void orc_unpack_row(const uint32_t* w, int64_t K, int64_t n, uint8_t* out) {
    const uint32_t* row = w + n * (K / 8);
    for (int64_t j = 0; j < K / 8; ++j) {
        uint32_t word = row[j];
        for (int i = 0; i < 8; ++i) out[8 * j + i] = (uint8_t)((word >> (4 * i)) & 0xFu);
    }
}

/*
 * y[m, n] = bf16( sum_k x[m,k] * (s[n,g] * q[n,k] + b[n,g]) ),  g = k / 64.
 * x: bf16 [M, K]; w: u32 [N, K/8]; s, b: bf16 [N, K/64]; y: bf16 [M, N].
 * If y_f32 is non-NULL the unrounded double sum is also stored (as float).
 *
 * Each group dot sum(q * x) is exact in double (every product q * x has at most 12
 * significant bits; 64 of them fit in 53 bits unless the group's activations span more
 * than ~2^35 in magnitude), so the order of its additions does not matter and the
 * vectorised path below returns the same bits as the scalar one. Groups are then
 * combined in double as acc += s * dot + b * xsum, in group order, in both paths.
 */
static void qmm_scalar(const float* xf, const double* xsum, int64_t M, int64_t K, const uint32_t* w,
                       const uint16_t* s, const uint16_t* b, int64_t N, uint16_t* y, float* y_f32) {
    const int64_t G = K / 64;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const uint32_t* row = w + n * (K / 8);
        float q[64];
        for (int64_t m = 0; m < M; ++m) {
            double acc = 0.0;
            const float* xr = xf + m * K;
            for (int64_t g = 0; g < G; ++g) {
                for (int j = 0; j < 8; ++j) {
                    uint32_t word = row[g * 8 + j];
                    for (int i = 0; i < 8; ++i) q[8 * j + i] = (float)((word >> (4 * i)) & 0xFu);
                }
                double dot = 0.0;
                const float* xg = xr + g * 64;
                for (int k = 0; k < 64; ++k) dot += (double)(q[k] * xg[k]);
                acc += (double)bf2f(s[n * G + g]) * dot + (double)bf2f(b[n * G + g]) * xsum[m * G + g];
            }
            y[m * N + n] = d2bf(acc);
            if (y_f32) y_f32[m * N + n] = (float)acc;
        }
    }
}

#if defined(__x86_64__) && defined(__GNUC__)
#include <immintrin.h>
#define ORC_HAVE_AVX2 1
__attribute__((target("avx2,fma"))) static void qmm_avx2(const double* xd, const double* xsum, int64_t M,
                                                          int64_t K, const uint32_t* w, const uint16_t* s,
                                                          const uint16_t* b, int64_t N, uint16_t* y,
                                                          float* y_f32) {
    const int64_t G = K / 64;
    double* accs = NULL;
#pragma omp parallel private(accs)
    {
        accs = (double*)malloc(sizeof(double) * (size_t)M);
        const __m256i shifts = _mm256_setr_epi32(0, 4, 8, 12, 16, 20, 24, 28);
        const __m256i fifteen = _mm256_set1_epi32(15);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            const uint32_t* row = w + n * (K / 8);
            for (int64_t m = 0; m < M; ++m) accs[m] = 0.0;
            /* four groups at a time: their dots reduce together (exact sums, so the
               reduction order is free) and s * dot + b * xsum is formed lane-wise with
               the scalar path's roundings; the four terms then enter acc in group order */
            for (int64_t g0 = 0; g0 < G; g0 += 4) {
                const int ng = (G - g0) < 4 ? (int)(G - g0) : 4;
                __m256d q[4][16];
                for (int gg = 0; gg < ng; ++gg)
                    for (int j = 0; j < 8; ++j) {
                        const __m256i c = _mm256_and_si256(
                            _mm256_srlv_epi32(_mm256_set1_epi32((int)row[(g0 + gg) * 8 + j]), shifts), fifteen);
                        q[gg][2 * j] = _mm256_cvtepi32_pd(_mm256_castsi256_si128(c));
                        q[gg][2 * j + 1] = _mm256_cvtepi32_pd(_mm256_extracti128_si256(c, 1));
                    }
                double sg[4] = {0, 0, 0, 0}, bg[4] = {0, 0, 0, 0};
                for (int gg = 0; gg < ng; ++gg) {
                    sg[gg] = (double)bf2f(s[n * G + g0 + gg]);
                    bg[gg] = (double)bf2f(b[n * G + g0 + gg]);
                }
                const __m256d sv = _mm256_loadu_pd(sg), bv = _mm256_loadu_pd(bg);
                for (int64_t m = 0; m < M; ++m) {
                    __m256d t[4];
                    for (int gg = 0; gg < 4; ++gg) {
                        if (gg >= ng) {
                            t[gg] = _mm256_setzero_pd();
                            continue;
                        }
                        const double* xg = xd + m * K + (g0 + gg) * 64;
                        __m256d a0 = _mm256_setzero_pd(), a1 = _mm256_setzero_pd();
                        for (int i = 0; i < 16; i += 2) {
                            a0 = _mm256_fmadd_pd(q[gg][i], _mm256_loadu_pd(xg + 4 * i), a0);
                            a1 = _mm256_fmadd_pd(q[gg][i + 1], _mm256_loadu_pd(xg + 4 * i + 4), a1);
                        }
                        t[gg] = _mm256_add_pd(a0, a1);
                    }
                    const __m256d h01 = _mm256_hadd_pd(t[0], t[1]);  /* t0[0]+t0[1], t1[0]+t1[1], t0[2]+t0[3], t1[2]+t1[3] */
                    const __m256d h23 = _mm256_hadd_pd(t[2], t[3]);
                    const __m256d dots = _mm256_add_pd(_mm256_permute2f128_pd(h01, h23, 0x20),
                                                       _mm256_permute2f128_pd(h01, h23, 0x31));
                    double xs[4] = {0, 0, 0, 0};
                    for (int gg = 0; gg < ng; ++gg) xs[gg] = xsum[m * G + g0 + gg];
                    double terms[4];
                    _mm256_storeu_pd(terms, _mm256_add_pd(_mm256_mul_pd(sv, dots),
                                                          _mm256_mul_pd(bv, _mm256_loadu_pd(xs))));
                    for (int gg = 0; gg < ng; ++gg) accs[m] += terms[gg];
                }
            }
            for (int64_t m = 0; m < M; ++m) {
                y[m * N + n] = d2bf(accs[m]);
                if (y_f32) y_f32[m * N + n] = (float)accs[m];
            }
        }
        free(accs);
    }
}
#endif

void orc_qmm(const uint16_t* x, int64_t M, int64_t K, const uint32_t* w,
             const uint16_t* s, const uint16_t* b, int64_t N, uint16_t* y,
             float* y_f32, int nthreads) {
    set_threads(nthreads);
    const int64_t G = K / 64;
    float* xf = (float*)malloc(sizeof(float) * (size_t)(M * K));
    double* xsum = (double*)malloc(sizeof(double) * (size_t)(M * G));
    for (int64_t i = 0; i < M * K; ++i) xf[i] = bf2f(x[i]);
    for (int64_t m = 0; m < M; ++m)
        for (int64_t g = 0; g < G; ++g) {
            double acc = 0.0;
            for (int k = 0; k < 64; ++k) acc += xf[m * K + g * 64 + k];
            xsum[m * G + g] = acc;
        }
#ifdef ORC_HAVE_AVX2
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && !getenv("ORC_SCALAR")) {
        double* xd = (double*)malloc(sizeof(double) * (size_t)(M * K));
        for (int64_t i = 0; i < M * K; ++i) xd[i] = (double)xf[i];
        qmm_avx2(xd, xsum, M, K, w, s, b, N, y, y_f32);
        free(xd);
        free(xf);
        free(xsum);
        return;
    }
#endif
    qmm_scalar(xf, xsum, M, K, w, s, b, N, y, y_f32);
    free(xf);
    free(xsum);
}

/*
 * Throughput-oriented variant used as the timed CPU baseline: the same
 * definition with float group dots and float accumulation (what a tuned CPU
 * kernel does), vectorised with AVX2/FMA where the host has it. Parity tests
 * use orc_qmm.
 */
#ifdef ORC_HAVE_AVX2
__attribute__((target("avx2,fma"))) static void qmv_fast_avx2(const float* xf, const float* xsum, int64_t K,
                                                               const uint32_t* w, const uint16_t* s,
                                                               const uint16_t* b, int64_t N, uint16_t* y) {
    const int64_t G = K / 64;
    /* x in the order the codes unpack: word j of a group gives codes 8j + i for lanes
       i = 0..7, so lane i of chunk j multiplies x[g * 64 + 8j + i] (no permutation) */
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const uint32_t* row = w + n * (K / 8);
        const __m256i shifts = _mm256_setr_epi32(0, 4, 8, 12, 16, 20, 24, 28);
        const __m256i fifteen = _mm256_set1_epi32(15);
        float acc = 0.f;
        for (int64_t g = 0; g < G; ++g) {
            __m256 d0 = _mm256_setzero_ps(), d1 = _mm256_setzero_ps();
            const float* xg = xf + g * 64;
            for (int j = 0; j < 8; j += 2) {
                const __m256i c0 = _mm256_and_si256(_mm256_srlv_epi32(_mm256_set1_epi32((int)row[g * 8 + j]), shifts),
                                                    fifteen);
                const __m256i c1 = _mm256_and_si256(
                    _mm256_srlv_epi32(_mm256_set1_epi32((int)row[g * 8 + j + 1]), shifts), fifteen);
                d0 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(c0), _mm256_loadu_ps(xg + 8 * j), d0);
                d1 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(c1), _mm256_loadu_ps(xg + 8 * j + 8), d1);
            }
            const __m256 t = _mm256_add_ps(d0, d1);
            __m128 h = _mm_add_ps(_mm256_castps256_ps128(t), _mm256_extractf128_ps(t, 1));
            h = _mm_add_ps(h, _mm_movehl_ps(h, h));
            h = _mm_add_ss(h, _mm_movehdup_ps(h));
            const float dot = _mm_cvtss_f32(h);
            acc += bf2f(s[n * G + g]) * dot + bf2f(b[n * G + g]) * xsum[g];
        }
        y[n] = f2bf(acc);
    }
}
#endif

void orc_qmv_fast(const uint16_t* x, int64_t K, const uint32_t* w,
                  const uint16_t* s, const uint16_t* b, int64_t N, uint16_t* y,
                  int nthreads) {
    set_threads(nthreads);
    const int64_t G = K / 64;
    float* xf = (float*)malloc(sizeof(float) * (size_t)K);
    float* xsum = (float*)malloc(sizeof(float) * (size_t)G);
    for (int64_t k = 0; k < K; ++k) xf[k] = bf2f(x[k]);
    for (int64_t g = 0; g < G; ++g) {
        float a = 0.f;
        for (int k = 0; k < 64; ++k) a += xf[g * 64 + k];
        xsum[g] = a;
    }
#ifdef ORC_HAVE_AVX2
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && !getenv("ORC_SCALAR")) {
        qmv_fast_avx2(xf, xsum, K, w, s, b, N, y);
        free(xf);
        free(xsum);
        return;
    }
#endif
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const uint32_t* row = w + n * (K / 8);
        float acc = 0.f;
        for (int64_t g = 0; g < G; ++g) {
            float dot = 0.f;
            for (int j = 0; j < 8; ++j) {
                uint32_t word = row[g * 8 + j];
                const float* xg = xf + g * 64 + j * 8;
                for (int i = 0; i < 8; ++i) dot += (float)((word >> (4 * i)) & 0xFu) * xg[i];
            }
            acc += bf2f(s[n * G + g]) * dot + bf2f(b[n * G + g]) * xsum[g];
        }
        y[n] = f2bf(acc);
    }
    free(xf);
    free(xsum);
}

/*
 * Attention for one sequence.
 *   q: bf16 [Lq, H, D]   (token-major rows, heads, head_dim)
 *   k, v: bf16 [Lk, Hkv, D]
 *   out: bf16 [Lq, H, D]
 * Query row i sits at absolute position q_pos0 + i, key row j at k_pos0 + j.
 * Key j is visible to query i iff kp <= qp and (window == 0 || kp > qp - window)
 * (forward.cc:345-374). Scores are multiplied by `scale` (the reference passes
 * 1.0). softcap > 0 applies softcap * tanh(score / softcap) before masking.
 * mode 0 = MLX CPU-stream rounding (bf16 scores, bf16 probabilities);
 * mode 1 = no intermediate rounding.
 */
void orc_sdpa(const uint16_t* q, const uint16_t* k, const uint16_t* v,
              int64_t Lq, int64_t Lk, int64_t H, int64_t Hkv, int64_t D,
              int64_t q_pos0, int64_t k_pos0, int64_t window, float scale,
              float softcap, int mode, uint16_t* out, int nthreads) {
    set_threads(nthreads);
    const int64_t rep = H / Hkv;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int64_t i = 0; i < Lq; ++i) {
        for (int64_t h = 0; h < H; ++h) {
            const int64_t hk = h / rep;
            const int64_t qp = q_pos0 + i;
            double* sc = (double*)malloc(sizeof(double) * (size_t)Lk);
            double* acc = (double*)calloc((size_t)D, sizeof(double));
            const uint16_t* qr = q + (i * H + h) * D;
            double mx = -INFINITY;
            for (int64_t j = 0; j < Lk; ++j) {
                const int64_t kp = k_pos0 + j;
                int vis = kp <= qp && (window == 0 || kp > qp - window);
                const uint16_t* kr = k + (j * Hkv + hk) * D;
                double dot = 0.0;
                for (int64_t d = 0; d < D; ++d) dot += (double)bf2f(qr[d]) * (double)bf2f(kr[d]);
                double sv = dot * (double)scale;
                if (mode == 0) sv = bf2f(d2bf(sv));
                if (softcap > 0.f) {
                    sv = (double)softcap * tanh(sv / (double)softcap);
                    if (mode == 0) sv = bf2f(d2bf(sv));
                }
                if (!vis) sv = -INFINITY;
                sc[j] = sv;
                if (sv > mx) mx = sv;
            }
            double den = 0.0;
            for (int64_t j = 0; j < Lk; ++j) {
                double e = (sc[j] == -INFINITY) ? 0.0 : exp(sc[j] - mx);
                sc[j] = e;
                den += e;
            }
            for (int64_t j = 0; j < Lk; ++j) {
                double p = sc[j] / den;
                if (mode == 0) p = bf2f(d2bf(p));
                if (p == 0.0) continue;
                const uint16_t* vr = v + (j * Hkv + hk) * D;
                for (int64_t d = 0; d < D; ++d) acc[d] += p * (double)bf2f(vr[d]);
            }
            uint16_t* orow = out + (i * H + h) * D;
            for (int64_t d = 0; d < D; ++d) orow[d] = d2bf(acc[d]);
            free(sc);
            free(acc);
        }
    }
}

/*
 * Seeded synthetic weights: a CPU restatement of the engine's on-device synthetic
 * loader, so the parity tests can rebuild the exact model the engine generated
 * (hyb_model_load_synthetic) without shipping a checkpoint. Every element is a pure
 * function of (seed, flat element index of the TP = 1 tensor):
 *   - codes: the low 32 bits of SplitMix64(seed * 0x100000001B3 + key);
 *   - normal deviates: ztab[top 16 bits of SplitMix64(key ^ 0xD1B54A32D192ED03)], where
 *     ztab holds the standard-normal quantiles at (i + 0.5) / 65536 (orc_normal_table);
 *   - scales bf16(|std * z|) with biases bf16(-8 * scale); norm vectors
 *     bf16(mean + std * z), multiply and add rounded separately.
 */
static inline uint64_t orc_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Wichura's AS 241 (PPND16, Applied Statistics 37:477-484, 1988): the inverse of the
   standard normal CDF in double precision. */
static double orc_ppnd16(double p) {
    const double q = p - 0.5;
    if (fabs(q) <= 0.425) {
        const double r = 0.180625 - q * q;
        const double num = ((((((2509.0809287301226727 * r + 33430.575583588128105) * r + 67265.770927008700853) * r +
                                45921.953931549871457) * r + 13731.693765509461125) * r + 1971.5909503065514427) * r +
                             133.14166789178437745) * r + 3.387132872796366608;
        const double den = ((((((5226.495278852545561 * r + 28729.085735721942674) * r + 39307.89580009271061) * r +
                                21213.794301586595867) * r + 5394.1960214247511077) * r + 687.1870074920579083) * r +
                             42.313330701600911252) * r + 1.0;
        return q * num / den;
    }
    double r = q < 0 ? p : 1.0 - p;
    r = sqrt(-log(r));
    double v;
    if (r <= 5.0) {
        r -= 1.6;
        v = (((((((7.7454501427834140764e-4 * r + 0.0227238449892691845833) * r + 0.24178072517745061177) * r +
                 1.27045825245236838258) * r + 3.64784832476320460504) * r + 5.7694972214606914055) * r +
              4.6303378461565452959) * r + 1.42343711074968357734) /
            (((((((1.05075007164441684324e-9 * r + 5.475938084995344946e-4) * r + 0.0151986665636164571966) * r +
                 0.14810397642748007459) * r + 0.68976733498510000455) * r + 1.6763848301838038494) * r +
              2.05319162663775882187) * r + 1.0);
    } else {
        r -= 5.0;
        v = (((((((2.01033439929228813265e-7 * r + 2.71155556874348757815e-5) * r + 0.0012426609473880784386) * r +
                 0.026532189526576123093) * r + 0.29656057182850489123) * r + 1.7848265399172913358) * r +
              5.4637849111641143699) * r + 6.6579046435011037772) /
            (((((((2.04426310338993978564e-15 * r + 1.4215117583164458887e-7) * r + 1.8463183175100546818e-5) * r +
                 7.868691311456132591e-4) * r + 0.0148753612908506148525) * r + 0.13692988092273580531) * r +
              0.59983220655588793769) * r + 1.0);
    }
    return q < 0 ? -v : v;
}

double orc_normal_quantile(double p) { return orc_ppnd16(p); }

void orc_normal_table(float* out) {
    for (int i = 0; i < 65536; ++i) out[i] = (float)orc_ppnd16((i + 0.5) / 65536.0);
}

/* words[i] for the [rows, cols] block at (row0, col0) of a [*, ld] u32 matrix */
void orc_synth_words(uint64_t seed, int64_t rows, int64_t cols, int64_t ld, int64_t row0, int64_t col0,
                     uint32_t* out, int nthreads) {
    set_threads(nthreads);
    const uint64_t base = seed * 0x100000001B3ull;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c)
            out[r * cols + c] = (uint32_t)orc_mix64(base + (uint64_t)((row0 + r) * ld + col0 + c));
}

/* scales bf16(|std * z|) and biases bf16(-8 * scale) for a [rows, cols] block */
void orc_synth_sb(uint64_t seed, int64_t rows, int64_t cols, int64_t ld, int64_t row0, int64_t col0, float stdv,
                  const float* ztab, uint16_t* s, uint16_t* b, int nthreads) {
    set_threads(nthreads);
    const uint64_t base = seed * 0x100000001B3ull;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) {
            const uint64_t key = base + (uint64_t)((row0 + r) * ld + col0 + c);
            const float z = ztab[orc_mix64(key ^ 0xD1B54A32D192ED03ull) >> 48];
            const uint16_t sv = f2bf(fabsf(stdv * z));
            s[r * cols + c] = sv;
            b[r * cols + c] = f2bf(-8.0f * bf2f(sv));
        }
}

/* bf16(mean + std * z) for n consecutive keys */
void orc_synth_normal(uint64_t seed, int64_t n, float mean, float stdv, const float* ztab, uint16_t* out) {
    const uint64_t base = seed * 0x100000001B3ull;
    for (int64_t i = 0; i < n; ++i) {
        const float z = ztab[orc_mix64((base + (uint64_t)i) ^ 0xD1B54A32D192ED03ull) >> 48];
        const float prod = stdv * z;
        out[i] = f2bf(mean + prod);
    }
}
