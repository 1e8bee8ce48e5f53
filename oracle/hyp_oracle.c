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
 */
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
    free(xf);
    free(xsum);
}

/*
 * Throughput-oriented variant used as the timed CPU baseline: the same
 * definition with float group dots and float accumulation (what a tuned CPU
 * kernel would do). Parity tests use orc_qmm.
 */
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
