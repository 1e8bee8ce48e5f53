// Fused decode attention for one token: QK-norm + RoPE + KV-cache append + SDPA,
// one thread-block cluster per KV head.
//
// Replaces, for q_len == 1, the reference's per-token sequence in
// ForwardPass::attention (native/hyperion_mlx/src/forward.cc:394-420 norms and
// RoPE, :459-468 cache append, :474-495 cache read, :498-504 SDPA).
//
// Each cluster of CS CTAs (CS <= 8, portable) owns one KV head and its REP query
// heads; CTA rank c owns a contiguous slice of the n_keys cache positions and
// each of its 8 warps a contiguous sub-slice. A warp streams its K rows and then
// its V rows through its own ring of 2 KB shared-memory stages with bulk copies
// (one cp.async.bulk per cache row, so ring wrap-around of the cache costs
// nothing; up to 16 KB in flight per warp). Warps never wait for each other while
// streaming. The first stages are issued before the programmatic-dependent-launch
// wait: cache rows of earlier positions never depend on the previous kernel.
//   phase 0  every CTA normalises and rotates its REP query heads from the raw
//            projection row; the CTA owning the newest position also normalises /
//            rotates the new K, normalises the new V, appends both to the cache
//            slot pos % cap and keeps them in shared memory (that row is never
//            bulk-copied);
//   phase 1  scores s = bf16(q . k * scale) into shared memory; per-CTA max and
//            sum of exp, pushed into every CTA of the cluster (remote stores);
//   cluster barrier; each CTA forms the row's (M, L) from the pushed pairs in
//            rank order;
//   phase 2  p = bf16(exp(s - M) / L) in place, P V per warp, summed over warps;
//            the CTA pushes each output element's partial to the CTA that owns
//            that element's slice;
//   cluster barrier; each CTA sums the pushed partials of its slice in rank order
//            (deterministic) and writes bf16.
// Only remote stores cross CTAs (no remote loads wait on latency). The cluster
// barriers are hardware barriers; every mbarrier wait is bounded.
#include "kernels.h"
#include "tma.cuh"

#include <algorithm>
#include <cfloat>

namespace hyb {

__device__ int g_attn_wait_timeouts = 0;  // set if a stage wait gave up (never expected)

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxCluster = 8;
constexpr int kStageBytes = 2048;
constexpr int kMaxStages = 8;  // per warp
constexpr size_t kSmemLimit = 227 * 1024;

__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared-memory address of `p` in the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
    uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(p)), remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
    return remote;
}

__device__ __forceinline__ void dsmem_st(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void dsmem_st2(uint32_t addr, float a, float b) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
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

template <int PER>
__device__ __forceinline__ void load_row(const bf16* p, float (&o)[PER]) {
    if constexpr (PER == 2) {
        uint32_t v = *reinterpret_cast<const uint32_t*>(p);
        o[0] = __uint_as_float(v << 16);
        o[1] = __uint_as_float(v & 0xFFFF0000u);
    } else if constexpr (PER == 4) {
        uint2 v = *reinterpret_cast<const uint2*>(p);
        o[0] = __uint_as_float(v.x << 16);
        o[1] = __uint_as_float(v.x & 0xFFFF0000u);
        o[2] = __uint_as_float(v.y << 16);
        o[3] = __uint_as_float(v.y & 0xFFFF0000u);
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

// Sum each of the V per-lane values over the warp. Reduce-scatter by halves
// (log2 V exchange steps), then a plain butterfly over the remaining lane bits:
// V - 1 + log2(32 / V) shuffles instead of 5 V. Afterwards v[0] of lane l holds
// the total of value index (l / (32 / V)).
template <int V>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[V]) {
    const int lane = threadIdx.x & 31;
    static_assert(V >= 1 && V <= 32 && (V & (V - 1)) == 0, "V must be a power of two <= 32");
#pragma unroll
    for (int half = V / 2, off = 16; half >= 1; half /= 2, off /= 2) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
#pragma unroll
    for (int off = 16 / V; off >= 1; off /= 2) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    return v[0];
}

// Normalise one head row of the raw projection (optionally rotate) into `dst`
// (floats holding bf16-rounded values). One warp; elements e = lane + 32 i.
template <int PER>
__device__ void norm_rope_row(const bf16* src, const bf16* nw, const float* inv_freq, int pos, float eps,
                              bool rope, float* dst, bf16* cache_dst) {
    const int lane = threadIdx.x & 31;
    constexpr int HD = PER * 32;
    float v[PER];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        v[i] = bf2f(src[lane + 32 * i]);
        ss += v[i] * v[i];
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const float t = rbf(v[i] * inv);
        v[i] = nw ? rbf(t * bf2f(nw[lane + 32 * i])) : t;
    }
    if (rope) {
        constexpr int HP = PER / 2;
#pragma unroll
        for (int i = 0; i < HP; ++i) {
            const float f = inv_freq[lane + 32 * i];
            if (f != 0.f) {
                float sn, cs;
                sincosf(__fmul_rn(static_cast<float>(pos), f), &sn, &cs);
                const float x1 = v[i], x2 = v[i + HP];
                v[i] = rbf(x1 * cs - x2 * sn);
                v[i + HP] = rbf(x1 * sn + x2 * cs);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        dst[lane + 32 * i] = v[i];
        if (cache_dst) cache_dst[lane + 32 * i] = f2bf(v[i]);
    }
}

// Shared-memory plan (bytes): rings, mbarriers, then the float arrays below.
struct FusedLayout {
    int stages;
    size_t rings, bars, q_s, knew, vnew, wred, ml, allml, stat, o_w, recv, s_sc, total;
};

__host__ __device__ inline FusedLayout fused_layout(int hd, int rep, int chunk, int stages) {
    FusedLayout L;
    L.stages = stages;
    L.rings = 0;
    L.bars = static_cast<size_t>(kWarps) * stages * kStageBytes;
    size_t f = L.bars + 8 * kWarps * kMaxStages;  // float cursor in bytes
    auto take = [&](size_t floats) {
        const size_t at = f;
        f += 4 * ((floats + 1) & ~static_cast<size_t>(1));  // keep 8-byte alignment
        return at;
    };
    const size_t E = static_cast<size_t>(rep) * hd;
    L.q_s = take(E);
    L.knew = take(hd);
    L.vnew = take(hd);
    L.wred = take(static_cast<size_t>(kWarps) * rep);
    L.ml = take(2 * rep);
    L.allml = take(2 * static_cast<size_t>(kMaxCluster) * rep);
    L.stat = take(2 * rep);
    L.o_w = take(static_cast<size_t>(kWarps) * E);
    L.recv = take(E + kMaxCluster);
    L.s_sc = take(static_cast<size_t>(rep) * chunk);
    L.total = f;
    return L;
}

template <int PER, int REP>
__global__ void __launch_bounds__(kThreads) decode_attn_fused_kernel(const DecodeFusedParams p, int chunk,
                                                                     int stages) {
    constexpr int HD = PER * 32;
    constexpr int E = REP * HD;
    constexpr int ROWB = HD * 2;               // bytes of one cache row
    constexpr int RS = kStageBytes / ROWB;     // rows per stage: 4 / 8 / 16
    constexpr int U = 4;                       // keys per score batch
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const FusedLayout lay = fused_layout(HD, REP, chunk, stages);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + lay.bars);
    float* q_s = reinterpret_cast<float*>(smem_raw + lay.q_s);      // [REP][HD]
    float* knew = reinterpret_cast<float*>(smem_raw + lay.knew);    // [HD]
    float* vnew = reinterpret_cast<float*>(smem_raw + lay.vnew);    // [HD]
    float* wred = reinterpret_cast<float*>(smem_raw + lay.wred);    // [kWarps][REP]
    float* ml = reinterpret_cast<float*>(smem_raw + lay.ml);        // [REP][2] this CTA's (max, sum)
    float* allml = reinterpret_cast<float*>(smem_raw + lay.allml);  // [CS][REP][2] pushed by every CTA
    float* stat = reinterpret_cast<float*>(smem_raw + lay.stat);    // [REP][2] (M, 1/L) of the row
    float* o_w = reinterpret_cast<float*>(smem_raw + lay.o_w);      // [kWarps][E]
    float* recv = reinterpret_cast<float*>(smem_raw + lay.recv);    // [CS][per_cta] pushed partials
    float* s_sc = reinterpret_cast<float*>(smem_raw + lay.s_sc);    // [REP][chunk]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hk = blockIdx.y;
    const int CS = gridDim.x;
    const uint32_t rank = cluster_rank();
    const int j0 = static_cast<int>(rank) * chunk;
    const int j1 = min(p.n_keys, j0 + chunk);
    const int n = max(0, j1 - j0);
    const bool owns_newest = (j1 == p.n_keys) && n > 0;
    const int first_pos = p.pos - p.n_keys + 1;
    // this warp's keys [wb, we) and its items: K stages then V stages
    const int kw = (n + kWarps - 1) / kWarps;
    const int wb = j0 + min(n, warp * kw), we = j0 + min(n, warp * kw + kw);
    const int nb = (we - wb + RS - 1) / RS;
    const int items = 2 * nb;
    unsigned char* ring = smem_raw + static_cast<size_t>(warp) * stages * kStageBytes;
    const uint32_t bar0 = smem_u32(bars + warp * kMaxStages);

    cluster_arrive_relaxed();  // matched by the wait before the first remote store
    if (lane == 0) {
        for (int s = 0; s < stages; ++s) mbar_init(bar0 + 8 * s, 1);
        mbar_init_fence();
    }
    __syncwarp();

    // Item i < nb: K rows of stage-batch i; i >= nb: V rows of batch i - nb.
    // Called by the whole warp; lane r copies row r of the batch.
    auto issue = [&](int i) {
        const bool isv = i >= nb;
        const int b = isv ? i - nb : i;
        const int rb = wb + b * RS, re = min(we, rb + RS);
        const bool has_new = owns_newest && re == p.n_keys;
        const int s = i % stages;
        const uint32_t bar = bar0 + 8 * s;
        if (lane == 0) mbar_expect_tx(bar, static_cast<uint32_t>(re - rb - (has_new ? 1 : 0)) * ROWB);
        __syncwarp();
        const int j = rb + lane;
        if (j < re && !(has_new && j == p.n_keys - 1)) {
            const int slot = (first_pos + j) % p.cap;
            const bf16* base = isv ? p.v_cache : p.k_cache;
            bulk_g2s(smem_u32(ring + s * kStageBytes) + lane * ROWB,
                     base + (static_cast<size_t>(slot) * p.n_kv + hk) * HD, ROWB, bar);
        }
    };
    for (int i = 0; i < stages && i < items; ++i) issue(i);

    pdl_wait();
    // ---- phase 0: query heads of this KV head, and the new token's K/V
    const int q_col = hk * REP * HD;
    const int k_col = p.n_heads * HD + hk * HD;
    const int v_col = p.v_from_k ? k_col : p.n_heads * HD + p.n_kv * HD + hk * HD;
    for (int r = warp; r < REP; r += kWarps - 2)
        norm_rope_row<PER>(p.qkv + q_col + r * HD, p.q_norm, p.inv_freq, p.pos, p.eps, true, q_s + r * HD,
                           nullptr);
    if (owns_newest) {
        const int slot = p.pos % p.cap;
        if (warp == kWarps - 1)
            norm_rope_row<PER>(p.qkv + k_col, p.k_norm, p.inv_freq, p.pos, p.eps, true, knew,
                               p.k_cache + (static_cast<size_t>(slot) * p.n_kv + hk) * HD);
        if (warp == kWarps - 2)
            norm_rope_row<PER>(p.qkv + v_col, nullptr, p.inv_freq, p.pos, p.eps, false, vnew,
                               p.v_cache + (static_cast<size_t>(slot) * p.n_kv + hk) * HD);
    }
    __syncthreads();

    uint32_t phase_bits = 0;  // one parity bit per stage
    bool waits_ok = true;
    auto wait_item = [&](int i) {
        const int s = i % stages;
        if (!mbar_wait_bounded(bar0 + 8 * s, (phase_bits >> s) & 1u)) waits_ok = false;
        phase_bits ^= 1u << s;
        return static_cast<const unsigned char*>(ring + s * kStageBytes);
    };
    auto release_item = [&](int i) {
        if (i + stages < items) {
            fence_proxy_async();  // this lane's reads of the stage precede the next copy into it
            __syncwarp();
            issue(i + stages);
        }
    };

    // ---- phase 1: scores of this warp's keys
    {
        float q[REP][PER];
#pragma unroll
        for (int r = 0; r < REP; ++r)
#pragma unroll
            for (int e = 0; e < PER; ++e) q[r][e] = q_s[r * HD + lane * PER + e];
        for (int b = 0; b < nb; ++b) {
            const unsigned char* st = wait_item(b);
            const int rb = wb + b * RS;
#pragma unroll
            for (int u0 = 0; u0 < RS; u0 += U) {
                float d[U * REP];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int j = rb + u0 + u;
                    float kv[PER];
                    if (owns_newest && j == p.n_keys - 1) {
#pragma unroll
                        for (int e = 0; e < PER; ++e) kv[e] = knew[lane * PER + e];
                    } else {
                        // rows past this warp's keys hold stale bytes; their scores are discarded
                        load_row<PER>(reinterpret_cast<const bf16*>(st + (u0 + u) * ROWB) + lane * PER, kv);
                    }
#pragma unroll
                    for (int h = 0; h < REP; ++h) {
                        float acc = 0.f;
#pragma unroll
                        for (int e = 0; e < PER; ++e) acc = fmaf(q[h][e], kv[e], acc);
                        d[u * REP + h] = acc;
                    }
                }
                const float tot = warp_reduce_scatter<U * REP>(d);
                constexpr int LPV = 32 / (U * REP);  // lanes per value after the reduce-scatter
                if (lane % LPV == 0) {
                    const int idx = lane / LPV;
                    const int j = rb + u0 + idx / REP;
                    if (j < we) s_sc[(idx % REP) * chunk + (j - j0)] = score_round(tot, p.scale, p.softcap, p.rounding);
                }
            }
            release_item(b);
        }
    }
    __syncthreads();
    // ---- per-head max and sum of exp over this CTA's keys
#pragma unroll
    for (int r = 0; r < REP; ++r) {
        float m = -FLT_MAX;
        for (int i = threadIdx.x; i < n; i += kThreads) m = fmaxf(m, s_sc[r * chunk + i]);
        m = warp_max(m);
        if (lane == 0) wred[warp * REP + r] = m;
    }
    __syncthreads();
    if (threadIdx.x < REP) {
        float m = -FLT_MAX;
        for (int w = 0; w < kWarps; ++w) m = fmaxf(m, wred[w * REP + threadIdx.x]);
        ml[2 * threadIdx.x] = m;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < REP; ++r) {
        const float m = ml[2 * r];
        float l = 0.f;
        for (int i = threadIdx.x; i < n; i += kThreads) l += expf(s_sc[r * chunk + i] - m);
        l = warp_sum(l);
        if (lane == 0) wred[warp * REP + r] = l;
    }
    __syncthreads();
    if (threadIdx.x < REP) {
        float l = 0.f;
        for (int w = 0; w < kWarps; ++w) l += wred[w * REP + threadIdx.x];
        ml[2 * threadIdx.x + 1] = l;
    }
    __syncthreads();
    // every CTA of the cluster has started: its shared memory may now be written
    cluster_wait();
    if (static_cast<int>(threadIdx.x) < CS * REP) {
        const int c = threadIdx.x / REP, r = threadIdx.x % REP;
        dsmem_st2(dsmem_addr(&allml[(rank * REP + r) * 2], c), ml[2 * r], ml[2 * r + 1]);
    }
    cluster_sync();
    if (threadIdx.x < REP) {
        const int r = threadIdx.x;
        float M = -FLT_MAX;
        for (int c = 0; c < CS; ++c) M = fmaxf(M, allml[(c * REP + r) * 2]);
        float L = 0.f;
        for (int c = 0; c < CS; ++c) {
            const float lc = allml[(c * REP + r) * 2 + 1];
            if (lc > 0.f) L += lc * expf(allml[(c * REP + r) * 2] - M);
        }
        stat[2 * r] = M;
        stat[2 * r + 1] = 1.0f / L;
    }
    __syncthreads();
    // probabilities in place: p = exp(s - M) / L, bf16-rounded unless rounding mode 1
    for (int i = threadIdx.x; i < REP * n; i += kThreads) {
        const int r = i / n, k = i - r * n;
        const float e = expf(s_sc[r * chunk + k] - stat[2 * r]) * stat[2 * r + 1];
        s_sc[r * chunk + k] = (p.rounding == 0) ? rbf(e) : e;
    }
    __syncthreads();
    // ---- phase 2: P V over this warp's keys
    {
        float acc[REP][PER];
#pragma unroll
        for (int r = 0; r < REP; ++r)
#pragma unroll
            for (int e = 0; e < PER; ++e) acc[r][e] = 0.f;
        for (int b = 0; b < nb; ++b) {
            const unsigned char* st = wait_item(nb + b);
            const int rb = wb + b * RS;
            const int rows = min(RS, we - rb);
#pragma unroll 4
            for (int u = 0; u < rows; ++u) {
                const int j = rb + u;
                float vv[PER];
                if (owns_newest && j == p.n_keys - 1) {
#pragma unroll
                    for (int e = 0; e < PER; ++e) vv[e] = vnew[lane * PER + e];
                } else {
                    load_row<PER>(reinterpret_cast<const bf16*>(st + u * ROWB) + lane * PER, vv);
                }
#pragma unroll
                for (int h = 0; h < REP; ++h) {
                    const float pr = s_sc[h * chunk + (j - j0)];
#pragma unroll
                    for (int e = 0; e < PER; ++e) acc[h][e] = fmaf(pr, vv[e], acc[h][e]);
                }
            }
            release_item(nb + b);
        }
#pragma unroll
        for (int r = 0; r < REP; ++r)
#pragma unroll
            for (int e = 0; e < PER; ++e) o_w[warp * E + r * HD + lane * PER + e] = acc[r][e];
    }
    __syncthreads();
    // ---- sum over warps, push each element's partial to the CTA owning its slice
    const int per_cta = (E + CS - 1) / CS;
    for (int i = threadIdx.x; i < E; i += kThreads) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += o_w[w * E + i];
        const int owner = i / per_cta;
        dsmem_st(dsmem_addr(&recv[rank * per_cta + (i - owner * per_cta)], owner), v);
    }
    cluster_sync();
    // ---- this CTA's slice, summed in rank order
    const int e0 = static_cast<int>(rank) * per_cta, e1 = min(E, e0 + per_cta);
    for (int i = e0 + static_cast<int>(threadIdx.x); i < e1; i += kThreads) {
        float v = 0.f;
        for (int c = 0; c < CS; ++c) v += recv[c * per_cta + (i - e0)];
        p.out[static_cast<size_t>(hk * REP) * HD + i] = f2bf(v);
    }
    pdl_launch_dependents();
    if (!waits_ok && lane == 0) {
        atomicAdd(&g_attn_wait_timeouts, 1);
        // copies that never signalled may still land: wait (bounded) before the CTA exits
        for (int s = 0; s < stages; ++s) mbar_wait_bounded(bar0 + 8 * s, ((phase_bits >> s) & 1u) ^ 1u);
    }
}

struct FusedPlan {
    int cs = 0, chunk = 0, stages = 0;
    size_t smem = 0;
};

FusedPlan plan_fused(int hd, int rep, int n_keys) {
    FusedPlan f;
    f.cs = std::min(kMaxCluster, std::max(1, (n_keys + 127) / 128));
    f.chunk = (n_keys + f.cs - 1) / f.cs;
    f.cs = (n_keys + f.chunk - 1) / f.chunk;
    for (int s = kMaxStages; s >= 1; s /= 2) {
        const FusedLayout L = fused_layout(hd, rep, f.chunk, s);
        f.stages = s;
        f.smem = L.total;
        if (f.smem <= kSmemLimit) return f;
    }
    f.stages = 0;
    return f;
}

template <int PER, int REP>
void launch_fused_t(const DecodeFusedParams& p, cudaStream_t stream, bool pdl) {
    const FusedPlan f = plan_fused(PER * 32, REP, p.n_keys);
    if (f.stages == 0) throw ArgError("decode attention: too many keys for the shared-memory plan");
    auto kern = decode_attn_fused_kernel<PER, REP>;
    static int attr_dev = -1;
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        HYB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit)));
        attr_dev = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(f.cs, p.n_kv);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = f.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = f.cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    HYB_CUDA(cudaLaunchKernelEx(&cfg, kern, p, f.chunk, f.stages));
}

template <int PER>
void launch_fused_rep(const DecodeFusedParams& p, cudaStream_t stream, bool pdl) {
    switch (p.n_heads / p.n_kv) {
        case 1: launch_fused_t<PER, 1>(p, stream, pdl); break;
        case 2: launch_fused_t<PER, 2>(p, stream, pdl); break;
        case 4: launch_fused_t<PER, 4>(p, stream, pdl); break;
        case 8: launch_fused_t<PER, 8>(p, stream, pdl); break;
        default: throw ArgError("decode attention: GQA group must be 1, 2, 4 or 8");
    }
}

}  // namespace

bool decode_attn_fused_fits(int n_heads, int n_kv, int hd, int n_keys) {
    if (n_kv <= 0 || n_heads % n_kv != 0 || (hd != 64 && hd != 128 && hd != 256) || n_keys <= 0) return false;
    const int rep = n_heads / n_kv;
    if (rep != 1 && rep != 2 && rep != 4 && rep != 8) return false;
    return plan_fused(hd, rep, n_keys).stages > 0;
}

void launch_decode_attn_fused(const DecodeFusedParams& p, cudaStream_t stream, bool pdl) {
    if (p.n_keys <= 0 || p.n_kv <= 0 || p.n_heads % p.n_kv != 0 || p.pos < p.n_keys - 1 || p.cap < p.n_keys)
        throw ArgError("decode attention: bad shape");
    if ((p.n_heads / p.n_kv) * p.hd > 1024) throw ArgError("decode attention: GQA group x head_dim > 1024");
    if ((reinterpret_cast<uintptr_t>(p.k_cache) | reinterpret_cast<uintptr_t>(p.v_cache)) & 15)
        throw ArgError("decode attention: K/V caches must be 16-byte aligned");
    switch (p.hd) {
        case 64: launch_fused_rep<2>(p, stream, pdl); break;
        case 128: launch_fused_rep<4>(p, stream, pdl); break;
        case 256: launch_fused_rep<8>(p, stream, pdl); break;
        default: throw ArgError("decode attention: head_dim must be 64, 128 or 256");
    }
}

int64_t read_attn_wait_timeouts() {
    int a = 0;
    HYB_CUDA(cudaMemcpyFromSymbol(&a, g_attn_wait_timeouts, sizeof(int)));
    return a;
}

}  // namespace hyb
