// Seeded stochastic sampling of one post-softcap logit row on the device: the steps of the
// reference's ForwardPass::sample_stochastic (native/hyperion_mlx/src/forward.cc:191-322)
// without copying the row to the host.
//
// Reference order: logits *= 1/temperature; p = softmax (fp32); top-p keeps the smallest set
// of most probable tokens whose mass reaches top_p; min-p drops p < min_p * max p; top-k
// keeps the k largest of the remaining logits; softmax over the kept ones; a draw
// u = uniform_real_distribution<float>(0, sz) from std::mt19937_64(seed); the token is the
// first index whose running sum reaches u. Every filter keeps a prefix of one total order
// (logit descending; among equal logits the reference's sorts leave the order unspecified,
// this kernel takes lower indices first), so the kept set is the first
// m = min(m_top_p, m_min_p, k) tokens of that order. The kernel finds m with radix
// selections over order-preserving 32-bit keys of the scaled logits (integer count and
// fixed-point mass histograms, so every run takes the same decisions), then sums and
// searches the kept probabilities in index order.
//
// One CTA of 1024 threads; thread t owns a contiguous chunk of the row, so index-order
// sums and searches are a per-thread walk plus one block scan. The row is re-read from L2
// on every pass (no scratch memory). Also returns the top-8 raw logits (the step result's
// top_k_logprob sidecar, forward.cc:295-310).
#include "kernels.h"

#include <cfloat>

namespace hyb {

namespace {

constexpr int kST = 1024;  // threads
constexpr int kSW = kST / 32;

// ---- MT19937-64 (Matsumoto and Nishimura's 64-bit Mersenne Twister, the engine
// std::mt19937_64 specifies): the first output after seeding needs state words 0, 1 and
// 156 of the initialisation, one twist of word 0, and the tempering.
__device__ uint64_t mt64_first(uint64_t seed) {
    constexpr uint64_t kMult = 6364136223846793005ull;
    uint64_t x = seed, w0 = seed, w1 = 0, w156 = 0;
    for (uint64_t i = 1; i <= 156; ++i) {
        x = kMult * (x ^ (x >> 62)) + i;
        if (i == 1) w1 = x;
        if (i == 156) w156 = x;
    }
    const uint64_t y = (w0 & 0xFFFFFFFF80000000ull) | (w1 & 0x7FFFFFFFull);
    uint64_t z = w156 ^ (y >> 1) ^ ((y & 1ull) ? 0xB5026F5AA96619E9ull : 0ull);
    z ^= (z >> 29) & 0x5555555555555555ull;
    z ^= (z << 17) & 0x71D67FFFEDA60000ull;
    z ^= (z << 37) & 0xFFF7EEE000000000ull;
    z ^= z >> 43;
    return z;
}

// uniform_real_distribution<float>(0, b) as libstdc++ evaluates it: generate_canonical
// takes one 64-bit output, converts it to float (nearest), divides by 2^64 and clamps below
// 1; the result is that times b.
__device__ float uniform_draw(uint64_t seed, float b) {
    float r = __ull2float_rn(mt64_first(seed)) * 5.42101086242752217e-20f;  // 2^-64
    if (r >= 1.0f) r = 0.99999994f;                                          // nextafter(1, 0)
    return __fmul_rn(r, b);
}

// Monotone 32-bit key of a float (larger float, larger key).
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct Shared {
    unsigned long long hist[256];
    unsigned long long red[kSW];
    float fred[kSW];
    uint32_t sel_prefix;
    unsigned long long sel_above;
    int found;
    float cand_v[kSW * 8];
    uint32_t cand_i[kSW * 8];
};

__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v, Shared& sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) sh.red[warp] = v;
    __syncthreads();
    unsigned long long t = 0;
    for (int w = 0; w < kSW; ++w) t += sh.red[w];
    return t;
}

// Fixed-order float sum over the CTA (each thread's value, warp trees, warps in order).
__device__ __forceinline__ float block_sum_f(float v, Shared& sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) sh.fred[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < kSW; ++w) t += sh.fred[w];
    return t;
}

__device__ __forceinline__ float block_max_f(float v, Shared& sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) sh.fred[warp] = v;
    __syncthreads();
    float t = -FLT_MAX;
    for (int w = 0; w < kSW; ++w) t = fmaxf(t, sh.fred[w]);
    return t;
}

// Exclusive prefix (in thread order) of a per-thread u64 and the total.
__device__ __forceinline__ unsigned long long block_excl_u64(unsigned long long v, unsigned long long* total, Shared& sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    __syncthreads();
    if (lane == 31) sh.red[warp] = inc;
    __syncthreads();
    unsigned long long before = 0, all = 0;
    for (int w = 0; w < kSW; ++w) {
        if (w < warp) before += sh.red[w];
        all += sh.red[w];
    }
    *total = all;
    return before + inc - v;
}

// Exclusive prefix (thread order) of a per-thread float, fixed association: the warps'
// inclusive sums, then the warps' totals added in warp order.
__device__ __forceinline__ float block_excl_f(float v, float* total, Shared& sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    __syncthreads();
    if (lane == 31) sh.fred[warp] = inc;
    __syncthreads();
    float before = 0.f, all = 0.f;
    for (int w = 0; w < kSW; ++w) {
        if (w < warp) before += sh.fred[w];
        all += sh.fred[w];
    }
    *total = all;
    return before + (inc - v);
}

struct Row {
    const bf16* x;
    int n, lo, hi;  // this thread's chunk [lo, hi)
    float inv_t, M, Z;
    __device__ float lg(int i) const { return bf2f(x[i]) * inv_t; }
    __device__ float prob(float l) const { return expf(l - M) / Z; }
};

// Fixed-point mass of a probability (2^-40 units).
__device__ __forceinline__ unsigned long long mass_of(float p) {
    return static_cast<unsigned long long>(p * 1099511627776.0f);
}

// The key T such that weight(key > T) < target <= weight(key >= T), weights being counts
// (MASS = false) or fixed-point masses; *above = weight(key > T). Requires target <= total.
template <bool MASS>
__device__ uint32_t radix_select(const Row& r, unsigned long long target, unsigned long long* above, Shared& sh) {
    uint32_t prefix = 0;
    unsigned long long acc = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = threadIdx.x; b < 256; b += kST) sh.hist[b] = 0;
        __syncthreads();
        for (int i = r.lo; i < r.hi; ++i) {
            const float l = r.lg(i);
            const uint32_t k = fkey(l);
            if (shift < 24 && (k >> (shift + 8)) != (prefix >> (shift + 8))) continue;
            atomicAdd(&sh.hist[(k >> shift) & 255u], MASS ? mass_of(r.prob(l)) : 1ull);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int sel = 0;
            for (int b = 255; b >= 0; --b) {
                if (acc + sh.hist[b] >= target) {
                    sel = b;
                    break;
                }
                acc += sh.hist[b];
            }
            sh.sel_prefix = prefix | (static_cast<uint32_t>(sel) << shift);
            sh.sel_above = acc;
        }
        __syncthreads();
        prefix = sh.sel_prefix;
        acc = sh.sel_above;
        __syncthreads();
    }
    *above = acc;
    return prefix;
}

__device__ __forceinline__ bool better(float v, uint32_t i, float w, uint32_t j) { return v > w || (v == w && i < j); }

__global__ void __launch_bounds__(kST, 1) sample_kernel(const bf16* __restrict__ x, int n, SampleSpec spec,
                                                        SampleResult* out) {
    __shared__ Shared sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (n + kST - 1) / kST;
    Row r;
    r.x = x;
    r.n = n;
    r.lo = min(n, tid * per);
    r.hi = min(n, r.lo + per);
    r.inv_t = 1.0f / spec.temperature;
    pdl_wait();

    // ---- pass 1: max scaled logit; this thread's top-8 raw logits (value desc, index asc)
    float tv[8];
    uint32_t ti[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        tv[k] = -FLT_MAX;
        ti[k] = 0xFFFFFFFFu;
    }
    float mx = -FLT_MAX;
    for (int i = r.lo; i < r.hi; ++i) {
        const float v = bf2f(x[i]);
        mx = fmaxf(mx, v * r.inv_t);
        if (better(v, i, tv[7], ti[7])) {
            int k = 7;
            while (k > 0 && better(v, i, tv[k - 1], ti[k - 1])) {
                tv[k] = tv[k - 1];
                ti[k] = ti[k - 1];
                --k;
            }
            tv[k] = v;
            ti[k] = static_cast<uint32_t>(i);
        }
    }
    r.M = block_max_f(mx, sh);
    // top-8 of the CTA: each warp merges its lanes' lists, then warp 0 merges the warps'
    {
        // each lane offers the head of its list; the winner pops its head (constant
        // register indices: the list shifts down)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float bv = tv[0];
            uint32_t bi = ti[0];
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (bi == ti[0] && bi != 0xFFFFFFFFu) {
#pragma unroll
                for (int q = 0; q < 7; ++q) {
                    tv[q] = tv[q + 1];
                    ti[q] = ti[q + 1];
                }
                tv[7] = -FLT_MAX;
                ti[7] = 0xFFFFFFFFu;
            }
            if (lane == 0) {
                sh.cand_v[warp * 8 + k] = bv;
                sh.cand_i[warp * 8 + k] = bi;
            }
        }
    }
    __syncthreads();
    if (warp == 0) {
        // lane l holds warp l's sorted list; 8 rounds of a warp argmax over the list heads
        int head = 0;
        for (int k = 0; k < 8; ++k) {
            const float v = head < 8 ? sh.cand_v[lane * 8 + head] : -FLT_MAX;
            const uint32_t i = head < 8 ? sh.cand_i[lane * 8 + head] : 0xFFFFFFFFu;
            float bv = v;
            uint32_t bi = i;
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (bi == i && head < 8 && i != 0xFFFFFFFFu) ++head;
            if (lane == 0) {
                out->topk_idx[k] = bi;
                out->topk_val[k] = bv;
            }
        }
        if (lane == 0) out->topk_count = n < 8 ? n : 8;
    }

    // ---- pass 2: softmax normaliser of the scaled logits
    float z = 0.f;
    for (int i = r.lo; i < r.hi; ++i) z += expf(r.lg(i) - r.M);
    r.Z = block_sum_f(z, sh);

    // ---- the kept prefix length m of the (logit desc, index asc) order
    unsigned long long m = static_cast<unsigned long long>(n);
    if (spec.min_p > 0.f && spec.min_p < 1.f) {
        const float thr = spec.min_p * (1.0f / r.Z);  // the largest probability is exp(0) / Z
        unsigned long long c = 0;
        for (int i = r.lo; i < r.hi; ++i) c += r.prob(r.lg(i)) >= thr ? 1ull : 0ull;
        m = min(m, block_sum_u64(c, sh));
    }
    if (spec.top_p > 0.f && spec.top_p < 1.f) {
        unsigned long long tot = 0;
        for (int i = r.lo; i < r.hi; ++i) tot += mass_of(r.prob(r.lg(i)));
        tot = block_sum_u64(tot, sh);
        const unsigned long long target = mass_of(spec.top_p);
        if (target <= tot && target > 0) {
            unsigned long long mass_gt = 0;
            const uint32_t T = radix_select<true>(r, target, &mass_gt, sh);
            unsigned long long c_gt = 0, c_eq = 0;
            float l_eq = 0.f;
            for (int i = r.lo; i < r.hi; ++i) {
                const float l = r.lg(i);
                const uint32_t k = fkey(l);
                c_gt += k > T ? 1ull : 0ull;
                if (k == T) {
                    ++c_eq;
                    l_eq = l;
                }
            }
            c_gt = block_sum_u64(c_gt, sh);
            c_eq = block_sum_u64(c_eq, sh);
            // every tied token has the same mass; the nucleus takes as few as reach top_p
            const float lt = block_max_f(c_eq ? l_eq : -FLT_MAX, sh);
            const unsigned long long me = mass_of(r.prob(lt));
            unsigned long long take = me ? (target - mass_gt + me - 1) / me : c_eq;
            take = max(1ull, min(take, c_eq));
            m = min(m, c_gt + take);
        }
    }
    if (spec.top_k > 0) m = min(m, static_cast<unsigned long long>(spec.top_k));
    if (m < 1) m = 1;
    uint32_t K = 0;      // the m-th key; keys above it are kept, and the first `ties` equal to it
    unsigned long long ties = 0;
    const bool all = m >= static_cast<unsigned long long>(n);
    if (!all) {
        unsigned long long c_gt = 0;
        K = radix_select<false>(r, m, &c_gt, sh);
        ties = m - c_gt;
    }

    // ---- sz: the kept tokens' exp(l - M) summed in index order
    unsigned long long my_ties = 0;
    if (!all)
        for (int i = r.lo; i < r.hi; ++i) my_ties += fkey(r.lg(i)) == K ? 1ull : 0ull;
    unsigned long long ties_total = 0;
    const unsigned long long tie0 = block_excl_u64(my_ties, &ties_total, sh);
    float part = 0.f;
    {
        unsigned long long tr = tie0;
        for (int i = r.lo; i < r.hi; ++i) {
            const float l = r.lg(i);
            bool keep = true;
            if (!all) {
                const uint32_t k = fkey(l);
                keep = k > K || (k == K && tr++ < ties);
            }
            part += keep ? expf(l - r.M) : 0.f;
        }
    }
    float sz = 0.f;
    const float before = block_excl_f(part, &sz, sh);
    // ---- the draw and the inverse-CDF search (first index whose running sum reaches u)
    const float u = uniform_draw(spec.seed, sz);
    if (tid == 0) sh.found = n - 1;  // a draw past the rounded total takes the last index
    __syncthreads();
    // the running sum at index i of thread t's chunk is before_t + (its chunk's sum up to
    // i, from zero), which ends at before_t + part_t; every thread that reaches u searches
    // and the smallest index wins
    if (r.lo < r.hi && u <= before + part) {
        float c = 0.f;
        unsigned long long tr = tie0;
        for (int i = r.lo; i < r.hi; ++i) {
            const float l = r.lg(i);
            bool keep = true;
            if (!all) {
                const uint32_t k = fkey(l);
                keep = k > K || (k == K && tr++ < ties);
            }
            c += keep ? expf(l - r.M) : 0.f;
            if (u <= before + c) {
                atomicMin(&sh.found, i);
                break;
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        out->token = static_cast<uint32_t>(sh.found);
        out->logit = bf2f(x[sh.found]);
        out->kept = static_cast<uint32_t>(m);
        out->u = u;
        out->sz = sz;
    }
}

}  // namespace

void launch_sample(const bf16* logits, int n, const SampleSpec& spec, SampleResult* out, cudaStream_t stream) {
    if (n < 1) throw ArgError("sampler: empty logit row");
    if (!(spec.temperature > 0.f)) throw ArgError("sampler: temperature must be > 0");
    sample_kernel<<<1, kST, 0, stream>>>(logits, n, spec, out);
    HYB_LAUNCH_CHECK("sample_kernel");
}

}  // namespace hyb
