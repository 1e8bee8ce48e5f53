// Gemma sliding-window / global attention over the BF16 KV caches.
//
// Replaces mx::fast::scaled_dot_product_attention(q, k, v, scale=1.0, bool mask)
// at native/hyperion_mlx/src/forward.cc:498-504 together with the cache reads
// that feed it (forward.cc:438-495; kv_cache.cc:251-265).
//
// Semantics (rounding = 0) are those of MLX's CPU-stream evaluation of that op:
// scores = bf16(q . k * scale); masked keys drop out; p = bf16(softmax_fp32(scores));
// out = bf16(sum_j p_j v_j) with fp32 accumulation. Because the probabilities are
// normalised BEFORE the bf16 rounding, both kernels below are two-pass.
//
// Decode (one query token, split-K over the cache):
//   kernel 1 (scores): CTA = (kv head, key split); each warp streams keys (one
//     128-bit load per lane at hd = 256), computes the scores of every query head
//     of the GQA group, stores them to scratch and emits the split's (max, sum exp).
//   kernel 2 (pv): CTA = (kv head, key split); combines the per-split (max, sum)
//     into the row's normaliser, rebuilds p = bf16(exp(s - M) / L) and accumulates
//     p * v; the last CTA of each kv head (atomic ticket) sums the split partials in
//     split order (deterministic) and writes bf16.
//   K and V are each read exactly once; the score round trip is H / (Hkv * hd) of
//   the K bytes (0.8% at 16 / (8 * 256)).
// The cache is a ring: position p lives in slot p % cap (a global cache has
// cap >= committed so the modulo is the identity there).
//
// Prefill (many query tokens): CTA = (64 query rows, head); pass 1 computes the
// row max and sum with mma.sync over the visible key blocks, pass 2 recomputes
// the scores, forms bf16 probabilities and accumulates P V on the tensor cores.
#include "kernels.h"

#include <algorithm>
#include <cfloat>
#include <mutex>

namespace hyb {

// Fixed scratch for hyb_sdpa_decode_noalloc (see launch_decode_attn_noalloc below).
// Every GPU that loads this library holds these bytes until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kDecThreads = 256;
constexpr int kMaxSplits = 64;
constexpr int kMaxRep = 8;

struct DecodeScratch {
    float* scores;    // [H][max_keys]
    float* ml;        // [H][kMaxSplits][2]
    float* opart;     // [kMaxSplits][H][hd]
    unsigned* tickets;  // [n_kv]
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

DecodeScratch carve(void* base, int H, int n_kv, int hd, int max_keys) {
    char* p = static_cast<char*>(base);
    DecodeScratch s;
    s.tickets = reinterpret_cast<unsigned*>(p);
    p += align256(sizeof(unsigned) * n_kv);
    s.ml = reinterpret_cast<float*>(p);
    p += align256(sizeof(float) * H * kMaxSplits * 2);
    s.opart = reinterpret_cast<float*>(p);
    p += align256(sizeof(float) * kMaxSplits * H * hd);
    s.scores = reinterpret_cast<float*>(p);
    return s;
}

__device__ __forceinline__ float score_round(float dot, float scale, float cap, int rounding) {
    float s = dot * scale;
    if (rounding == 0) s = rbf(s);
    if (cap > 0.f) {
        s = cap * tanhf(s / cap);
        if (rounding == 0) s = rbf(s);
    }
    return s;
}

// Load `per` consecutive bf16 (per in {2,4,8,16}) starting at p into floats.
template <int PER>
__device__ __forceinline__ void load_row(const bf16* p, float (&o)[PER]) {
    if constexpr (PER == 2) {
        uint32_t v = *reinterpret_cast<const uint32_t*>(p);
        o[0] = __uint_as_float(v << 16);
        o[1] = __uint_as_float(v & 0xFFFF0000u);
    } else if constexpr (PER == 4) {
        uint2 v = *reinterpret_cast<const uint2*>(p);
        o[0] = __uint_as_float(v.x << 16); o[1] = __uint_as_float(v.x & 0xFFFF0000u);
        o[2] = __uint_as_float(v.y << 16); o[3] = __uint_as_float(v.y & 0xFFFF0000u);
    } else {
#pragma unroll
        for (int c = 0; c < PER / 8; ++c) {
            uint4 v = *reinterpret_cast<const uint4*>(p + 8 * c);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                o[8 * c + 2 * i] = __uint_as_float(w[i] << 16);
                o[8 * c + 2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
            }
        }
    }
}

template <int PER, int REP>
__global__ void __launch_bounds__(kDecThreads) decode_scores_kernel(DecodeAttnParams p, DecodeScratch sc,
                                                                    int n_splits, int chunk) {
    const int hk = blockIdx.x, split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = p.hd;
    const int j0 = split * chunk, j1 = min(p.n_keys, j0 + chunk);
    __shared__ float s_sc[REP][512];  // chunk <= 512
    __shared__ float s_red[REP][8];
    pdl_wait();
    float q[REP][PER];
#pragma unroll
    for (int r = 0; r < REP; ++r) load_row<PER>(p.q + static_cast<size_t>(hk * REP + r) * hd + lane * PER, q[r]);
    const int first_pos = p.last_pos - p.n_keys + 1;
    constexpr int U = 4;  // keys in flight per warp
    for (int jb = j0 + warp * U; jb < j1; jb += 8 * U) {
        float kv[U][PER];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = jb + u;
            if (j < j1) {
                const int slot = (first_pos + j) % p.cap;
                load_row<PER>(p.k_cache + (static_cast<size_t>(slot) * p.n_kv + hk) * hd + lane * PER, kv[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = jb + u;
#pragma unroll
            for (int r = 0; r < REP; ++r) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < PER; ++e) d = fmaf(q[r][e], kv[u][e], d);
                d = warp_sum(d);
                if (lane == 0 && j < j1) s_sc[r][j - j0] = score_round(d, p.scale, p.softcap, p.rounding);
            }
        }
    }
    __syncthreads();
    // per head: max and sum of exp over this split; also publish raw scores
    const int n = j1 - j0;
#pragma unroll
    for (int r = 0; r < REP; ++r) {
        float m = -FLT_MAX;
        for (int i = threadIdx.x; i < n; i += kDecThreads) m = fmaxf(m, s_sc[r][i]);
        m = warp_max(m);
        if (lane == 0) s_red[r][warp] = m;
        __syncthreads();
        m = -FLT_MAX;
#pragma unroll
        for (int w = 0; w < 8; ++w) m = fmaxf(m, s_red[r][w]);
        __syncthreads();
        float l = 0.f;
        const int h = hk * REP + r;
        for (int i = threadIdx.x; i < n; i += kDecThreads) {
            const float v = s_sc[r][i];
            l += expf(v - m);
            sc.scores[static_cast<size_t>(h) * p.n_keys + j0 + i] = v;
        }
        l = warp_sum(l);
        if (lane == 0) s_red[r][warp] = l;
        __syncthreads();
        if (threadIdx.x == 0) {
            float tot = 0.f;
            for (int w = 0; w < 8; ++w) tot += s_red[r][w];
            sc.ml[(static_cast<size_t>(h) * kMaxSplits + split) * 2 + 0] = (n > 0) ? m : -FLT_MAX;
            sc.ml[(static_cast<size_t>(h) * kMaxSplits + split) * 2 + 1] = (n > 0) ? tot : 0.f;
        }
        __syncthreads();
    }
    pdl_launch_dependents();
}

template <int PER, int REP>
__global__ void __launch_bounds__(kDecThreads) decode_pv_kernel(DecodeAttnParams p, DecodeScratch sc,
                                                                int n_splits, int chunk) {
    const int hk = blockIdx.x, split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = p.hd;
    const int j0 = split * chunk, j1 = min(p.n_keys, j0 + chunk);
    __shared__ float s_M[REP], s_invL[REP];
    static_assert(REP * PER * 32 <= 1024, "GQA group x head_dim above 1024");
    constexpr int kAcc = REP * PER * 32;  // per-warp REP * hd floats
    __shared__ float s_acc[8][kAcc];
    __shared__ unsigned s_ticket;
    pdl_wait();
    if (threadIdx.x < REP) {
        const int h = hk * REP + threadIdx.x;
        float M = -FLT_MAX;
        for (int s = 0; s < n_splits; ++s) M = fmaxf(M, sc.ml[(static_cast<size_t>(h) * kMaxSplits + s) * 2]);
        float L = 0.f;
        for (int s = 0; s < n_splits; ++s) {
            const float ms = sc.ml[(static_cast<size_t>(h) * kMaxSplits + s) * 2];
            const float ls = sc.ml[(static_cast<size_t>(h) * kMaxSplits + s) * 2 + 1];
            if (ls > 0.f) L += ls * expf(ms - M);
        }
        s_M[threadIdx.x] = M;
        s_invL[threadIdx.x] = 1.0f / L;
    }
    __syncthreads();
    float acc[REP][PER];
#pragma unroll
    for (int r = 0; r < REP; ++r)
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[r][e] = 0.f;
    const int first_pos = p.last_pos - p.n_keys + 1;
    constexpr int U = 4;
    for (int jb = j0 + warp * U; jb < j1; jb += 8 * U) {
        float vv[U][PER];
        float pr[U][REP];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = jb + u;
            if (j < j1) {
                const int slot = (first_pos + j) % p.cap;
                load_row<PER>(p.v_cache + (static_cast<size_t>(slot) * p.n_kv + hk) * hd + lane * PER, vv[u]);
#pragma unroll
                for (int r = 0; r < REP; ++r) {
                    const int h = hk * REP + r;
                    float e = expf(sc.scores[static_cast<size_t>(h) * p.n_keys + j] - s_M[r]) * s_invL[r];
                    pr[u][r] = (p.rounding == 0) ? rbf(e) : e;
                }
            } else {
#pragma unroll
                for (int e = 0; e < PER; ++e) vv[u][e] = 0.f;
#pragma unroll
                for (int r = 0; r < REP; ++r) pr[u][r] = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int r = 0; r < REP; ++r)
#pragma unroll
                for (int e = 0; e < PER; ++e) acc[r][e] = fmaf(pr[u][r], vv[u][e], acc[r][e]);
    }
    // reduce the 8 warps through shared memory, write this split's partial
    float* mine = &s_acc[warp][0];
#pragma unroll
    for (int r = 0; r < REP; ++r)
#pragma unroll
        for (int e = 0; e < PER; ++e) mine[r * hd + lane * PER + e] = acc[r][e];
    __syncthreads();
    for (int i = threadIdx.x; i < REP * hd; i += kDecThreads) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += s_acc[w][i];
        const int r = i / hd, e = i % hd;
        sc.opart[(static_cast<size_t>(split) * p.n_heads + hk * REP + r) * hd + e] = v;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(&sc.tickets[hk], 1u);
    __syncthreads();
    if (s_ticket != static_cast<unsigned>(n_splits - 1)) return;
    // last CTA for this kv head: deterministic split-ordered sum
    __threadfence();
    for (int i = threadIdx.x; i < REP * hd; i += kDecThreads) {
        const int r = i / hd, e = i % hd;
        float v = 0.f;
        for (int s = 0; s < n_splits; ++s)
            v += __ldcg(&sc.opart[(static_cast<size_t>(s) * p.n_heads + hk * REP + r) * hd + e]);
        p.out[static_cast<size_t>(hk * REP + r) * hd + e] = f2bf(v);
    }
    if (threadIdx.x == 0) sc.tickets[hk] = 0u;  // ready for the next launch
    pdl_launch_dependents();
}

void decode_plan(int n_kv, int n_keys, int& n_splits, int& chunk) {
    const int target = std::max(1, (2 * num_sms() + n_kv - 1) / n_kv);
    int s = std::min(target, kMaxSplits);
    chunk = std::max(32, (n_keys + s - 1) / s);
    chunk = std::min(chunk, 512);
    n_splits = (n_keys + chunk - 1) / chunk;
    if (n_splits > kMaxSplits) {
        chunk = (n_keys + kMaxSplits - 1) / kMaxSplits;
        n_splits = (n_keys + chunk - 1) / chunk;
    }
}

template <int PER, int REP>
void launch_decode_t(const DecodeAttnParams& p, const DecodeScratch& sc, cudaStream_t stream) {
    if constexpr (REP * PER * 32 > 1024) {
        // GQA group x head_dim above 1024 (rejected by the caller): not instantiated.
        throw ArgError("decode attention: GQA group x head_dim > 1024");
    } else {
    int n_splits, chunk;
    decode_plan(p.n_kv, p.n_keys, n_splits, chunk);
    if (chunk > 512) throw ArgError("decode attention: too many keys for the split plan");
    dim3 grid(p.n_kv, n_splits);
    decode_scores_kernel<PER, REP><<<grid, kDecThreads, 0, stream>>>(p, sc, n_splits, chunk);
    HYB_LAUNCH_CHECK("decode_scores_kernel");
    decode_pv_kernel<PER, REP><<<grid, kDecThreads, 0, stream>>>(p, sc, n_splits, chunk);
    HYB_LAUNCH_CHECK("decode_pv_kernel");
    }
}

template <int PER>
void launch_decode_rep(const DecodeAttnParams& p, const DecodeScratch& sc, cudaStream_t stream) {
    switch (p.n_heads / p.n_kv) {
        case 1: launch_decode_t<PER, 1>(p, sc, stream); break;
        case 2: launch_decode_t<PER, 2>(p, sc, stream); break;
        case 4: launch_decode_t<PER, 4>(p, sc, stream); break;
        case 8: launch_decode_t<PER, 8>(p, sc, stream); break;
        default: throw ArgError("decode attention: GQA group must be 1, 2, 4 or 8");
    }
}

// ============================================================================ prefill
constexpr int kPQ = 64;       // query rows per CTA (4 warps x 16)
constexpr int kPK = 64;       // keys per block
constexpr int kPThreads = 128;

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}

template <int HD>
struct PrefillSmem {
    static constexpr int LD = HD + 8;  // bf16 elements per row (16-byte pad)
    bf16 q[kPQ * LD];
    bf16 k[kPK * LD];
    bf16 v[kPK * LD];
};

template <int HD>
__device__ __forceinline__ void load_tile(bf16* dst, const bf16* src, int rows, int row_stride_elems,
                                          int valid_rows) {
    constexpr int LD = HD + 8;
    constexpr int vec_per_row = HD / 8;
    for (int i = threadIdx.x; i < rows * vec_per_row; i += kPThreads) {
        const int r = i / vec_per_row, c = i % vec_per_row;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < valid_rows) v = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * row_stride_elems + 8 * c);
        *reinterpret_cast<uint4*>(dst + r * LD + 8 * c) = v;
    }
}

// S = Q K^T for this warp's 16 rows x 64 keys.
template <int HD>
__device__ __forceinline__ void qk_tile(const PrefillSmem<HD>& sm, int warp, int lane, float (&s)[8][4]) {
    constexpr int LD = HD + 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD; kk += 16) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(a0, a1, a2, a3, &sm.q[(warp * 16 + (lane & 15)) * LD + kk + (lane >> 4) * 8]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t b0, b1, b2, b3;
            const int nrow = j * 16 + (lane & 7) + ((lane >> 4) << 3);
            ldsm_x4(b0, b1, b2, b3, &sm.k[nrow * LD + kk + ((lane >> 3) & 1) * 8]);
            mma_bf16_16816(s[2 * j], a0, a1, a2, a3, b0, b1);
            mma_bf16_16816(s[2 * j + 1], a0, a1, a2, a3, b2, b3);
        }
    }
}

template <int HD>
__global__ void __launch_bounds__(kPThreads) prefill_attn_kernel(const PrefillAttnParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PrefillSmem<HD>& sm = *reinterpret_cast<PrefillSmem<HD>*>(smem_raw);
    constexpr int LD = HD + 8;
    const int qb = blockIdx.x, h = blockIdx.y;
    const int hk = h / (p.n_heads / p.n_kv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int q0 = qb * kPQ;
    const int qrows = min(kPQ, p.Lq - q0);
    load_tile<HD>(sm.q, p.q + (static_cast<size_t>(q0) * p.n_heads + h) * HD, kPQ, p.n_heads * HD, qrows);

    // visible key index range for the whole block
    const int qp_lo = p.q_pos0 + q0, qp_hi = p.q_pos0 + q0 + qrows - 1;
    int j_lo = 0;
    if (p.window > 0) j_lo = max(0, qp_lo - p.window + 1 - p.k_pos0);
    const int j_hi = min(p.Lk, qp_hi - p.k_pos0 + 1);  // exclusive
    // this thread's two query rows
    const int r0 = warp * 16 + g, r1 = r0 + 8;
    const int qp0 = p.q_pos0 + q0 + r0, qp1 = p.q_pos0 + q0 + r1;

    float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.f, l1 = 0.f;
    auto visible = [&](int qp, int j) {
        const int kp = p.k_pos0 + j;
        return j < p.Lk && kp <= qp && (p.window == 0 || kp > qp - p.window);
    };
    // ---------------- pass 1: row max and sum
    for (int kb = j_lo; kb < j_hi; kb += kPK) {
        __syncthreads();
        load_tile<HD>(sm.k, p.k + (static_cast<size_t>(kb) * p.n_kv + hk) * HD, kPK, p.n_kv * HD, min(kPK, p.Lk - kb));
        __syncthreads();
        float s[8][4];
        qk_tile<HD>(sm, warp, lane, s);
        float mx0 = m0, mx1 = m1;
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int key = kb + j * 8 + 2 * t + (c & 1);
                const bool top = c < 2;
                float v = score_round(s[j][c], p.scale, p.softcap, p.rounding);
                if (!visible(top ? qp0 : qp1, key)) v = -FLT_MAX;
                s[j][c] = v;
                if (top) mx0 = fmaxf(mx0, v); else mx1 = fmaxf(mx1, v);
            }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            a0 += (s[j][0] == -FLT_MAX ? 0.f : expf(s[j][0] - mx0)) + (s[j][1] == -FLT_MAX ? 0.f : expf(s[j][1] - mx0));
            a1 += (s[j][2] == -FLT_MAX ? 0.f : expf(s[j][2] - mx1)) + (s[j][3] == -FLT_MAX ? 0.f : expf(s[j][3] - mx1));
        }
        a0 += __shfl_xor_sync(0xffffffffu, a0, 1);
        a0 += __shfl_xor_sync(0xffffffffu, a0, 2);
        a1 += __shfl_xor_sync(0xffffffffu, a1, 1);
        a1 += __shfl_xor_sync(0xffffffffu, a1, 2);
        l0 = (m0 == -FLT_MAX ? 0.f : l0 * expf(m0 - mx0)) + a0;
        l1 = (m1 == -FLT_MAX ? 0.f : l1 * expf(m1 - mx1)) + a1;
        m0 = mx0;
        m1 = mx1;
    }
    const float il0 = l0 > 0.f ? 1.0f / l0 : 0.f, il1 = l1 > 0.f ? 1.0f / l1 : 0.f;
    // ---------------- pass 2: probabilities and P V
    float o[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    for (int kb = j_lo; kb < j_hi; kb += kPK) {
        __syncthreads();
        load_tile<HD>(sm.k, p.k + (static_cast<size_t>(kb) * p.n_kv + hk) * HD, kPK, p.n_kv * HD, min(kPK, p.Lk - kb));
        load_tile<HD>(sm.v, p.v + (static_cast<size_t>(kb) * p.n_kv + hk) * HD, kPK, p.n_kv * HD, min(kPK, p.Lk - kb));
        __syncthreads();
        float s[8][4];
        qk_tile<HD>(sm, warp, lane, s);
        uint32_t pa[8][2];  // probabilities packed as bf16 pairs, in C-fragment order
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float pr[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int key = kb + j * 8 + 2 * t + (c & 1);
                const bool top = c < 2;
                float v = score_round(s[j][c], p.scale, p.softcap, p.rounding);
                float e = visible(top ? qp0 : qp1, key) ? expf(v - (top ? m0 : m1)) * (top ? il0 : il1) : 0.f;
                pr[c] = e;
            }
            pa[j][0] = pack_bf2(f2bf(pr[0]), f2bf(pr[1]));
            pa[j][1] = pack_bf2(f2bf(pr[2]), f2bf(pr[3]));
        }
        // O += P (16 x 64) * V (64 x HD)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // 16 keys per k-step
            const uint32_t a0 = pa[2 * kk][0], a1 = pa[2 * kk][1], a2 = pa[2 * kk + 1][0], a3 = pa[2 * kk + 1][1];
#pragma unroll
            for (int n = 0; n < HD / 16; ++n) {
                uint32_t b0, b1, b2, b3;
                // V is [key][hd]: a transposed ldmatrix yields the col-major B fragment
                const int krow = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                const int col = n * 16 + ((lane >> 4) << 3);
                ldsm_x4_t(b0, b1, b2, b3, &sm.v[krow * LD + col]);
                mma_bf16_16816(o[2 * n], a0, a1, a2, a3, b0, b1);
                mma_bf16_16816(o[2 * n + 1], a0, a1, a2, a3, b2, b3);
            }
        }
    }
    // store
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
        const int col = n * 8 + 2 * t;
        if (r0 < qrows) {
            *reinterpret_cast<__nv_bfloat162*>(p.out + (static_cast<size_t>(q0 + r0) * p.n_heads + h) * HD + col) =
                __floats2bfloat162_rn(o[n][0], o[n][1]);
        }
        if (r1 < qrows) {
            *reinterpret_cast<__nv_bfloat162*>(p.out + (static_cast<size_t>(q0 + r1) * p.n_heads + h) * HD + col) =
                __floats2bfloat162_rn(o[n][2], o[n][3]);
        }
    }
}

template <int HD>
void launch_prefill_t(const PrefillAttnParams& p, cudaStream_t stream) {
    const size_t smem = sizeof(PrefillSmem<HD>);
    static int attr_dev = -1;
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        HYB_CUDA(cudaFuncSetAttribute(prefill_attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
        attr_dev = dev;
    }
    dim3 grid((p.Lq + kPQ - 1) / kPQ, p.n_heads);
    prefill_attn_kernel<HD><<<grid, kPThreads, smem, stream>>>(p);
    HYB_LAUNCH_CHECK("prefill_attn_kernel");
}

}  // namespace

size_t decode_attn_scratch_bytes(int n_heads, int n_kv, int hd, int max_keys) {
    return align256(sizeof(unsigned) * n_kv) + align256(sizeof(float) * n_heads * kMaxSplits * 2) +
           align256(sizeof(float) * kMaxSplits * n_heads * hd) +
           align256(sizeof(float) * static_cast<size_t>(n_heads) * max_keys);
}

// Every shape check of the split-K decode attention except the scratch size (throws ArgError).
static void check_decode_attn_shape(const DecodeAttnParams& p) {
    if (p.n_keys <= 0 || p.n_kv <= 0 || p.n_heads % p.n_kv != 0) throw ArgError("decode attention: bad shape");
    if (p.n_heads / p.n_kv > kMaxRep) throw ArgError("decode attention: GQA group too large");
    if (p.n_keys > kMaxSplits * 512) throw ArgError("decode attention: more than 32768 keys");
    if ((p.n_heads / p.n_kv) * p.hd > 1024) throw ArgError("decode attention: GQA group x head_dim > 1024");
    if (p.hd != 64 && p.hd != 128 && p.hd != 256 && p.hd != 512)
        throw ArgError("decode attention: head_dim must be 64, 128, 256 or 512");
}

void launch_decode_attn(const DecodeAttnParams& p, cudaStream_t stream) {
    check_decode_attn_shape(p);
    if (p.scratch_bytes < decode_attn_scratch_bytes(p.n_heads, p.n_kv, p.hd, p.n_keys))
        throw ArgError("decode attention: scratch too small");
    DecodeScratch sc = carve(p.scratch, p.n_heads, p.n_kv, p.hd, p.n_keys);
    switch (p.hd) {
        case 64: launch_decode_rep<2>(p, sc, stream); break;
        case 128: launch_decode_rep<4>(p, sc, stream); break;
        case 256: launch_decode_rep<8>(p, sc, stream); break;
        case 512: launch_decode_rep<16>(p, sc, stream); break;
        default: throw ArgError("decode attention: head_dim must be 64, 128, 256 or 512");
    }
}

// Device address of g_decode_noalloc_scratch on the current device. Host code only
// sees a host-side stand-in for the symbol, so the device address is looked up
// once per device with cudaGetSymbolAddress (with that device current) and cached.
// A device reset (cudaDeviceReset) reloads the module, possibly elsewhere, and makes
// the cached address stale; this library does not reset devices.
static void* noalloc_scratch_on_current_device() {
    static std::mutex mu;
    static void* addr[64] = {};
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw ArgError("sdpa_decode_noalloc: device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        HYB_CUDA(cudaGetSymbolAddress(&p, g_decode_noalloc_scratch));
        addr[dev] = p;
    }
    return addr[dev];
}

size_t decode_attn_noalloc_limit_bytes() { return kNoAllocScratchBytes; }

void launch_decode_attn_noalloc(DecodeAttnParams p, cudaStream_t stream) {
    // a rejected call queues no GPU work: every check runs before the counters are cleared
    check_decode_attn_shape(p);
    const size_t need = decode_attn_scratch_bytes(p.n_heads, p.n_kv, p.hd, p.n_keys);
    if (need > kNoAllocScratchBytes)
        throw ArgError("sdpa_decode_noalloc: this call needs " + std::to_string(need) +
                       " bytes of scratch, above the fixed 8 MiB (8388608-byte) device buffer");
    void* scratch = noalloc_scratch_on_current_device();
    // The buffer keeps whatever the previous call left; the per-KV-head completion
    // counters must start at zero, so clear them for this call (no allocation).
    HYB_CUDA(cudaMemsetAsync(scratch, 0, align256(sizeof(unsigned) * p.n_kv), stream));
    p.scratch = scratch;
    p.scratch_bytes = kNoAllocScratchBytes;
    launch_decode_attn(p, stream);
}

void launch_prefill_attn(const PrefillAttnParams& p, cudaStream_t stream) {
    if (p.Lq <= 0) return;
    if (p.n_kv <= 0 || p.n_heads % p.n_kv != 0) throw ArgError("prefill attention: bad head counts");
    if (prefill_attn_tc_supported(p)) {
        launch_prefill_attn_tc(p, stream);
        return;
    }
    launch_prefill_attn_mma(p, stream);
}

void launch_prefill_attn_mma(const PrefillAttnParams& p, cudaStream_t stream) {
    if (p.Lq <= 0) return;
    if (p.n_kv <= 0 || p.n_heads % p.n_kv != 0) throw ArgError("prefill attention: bad head counts");
    switch (p.hd) {
        case 64: launch_prefill_t<64>(p, stream); break;
        case 128: launch_prefill_t<128>(p, stream); break;
        case 256: launch_prefill_t<256>(p, stream); break;
        default: throw ArgError("prefill attention: head_dim must be 64, 128 or 256");
    }
}

}  // namespace hyb
