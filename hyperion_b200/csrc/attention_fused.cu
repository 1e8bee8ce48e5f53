// Fused decode attention for one token: QK-norm + RoPE + KV-cache append + SDPA,
// one thread-block cluster per KV head.
//
// Replaces, for q_len == 1, the reference's per-token sequence in
// ForwardPass::attention (native/hyperion_mlx/src/forward.cc:394-420 norms and
// RoPE, :459-468 cache append, :474-495 cache read, :498-504 SDPA).
//
// Each cluster of CS CTAs (CS <= 16: above 8 only where the occupancy query says that
// many clusters of that size are resident at once) owns one KV head and its REP query
// heads (of one sequence: a batched launch adds gridDim.z = sequences and reads each
// sequence's caches, position and tensor maps from a DecodeSeq array; CS then shrinks
// so that the launch fits the SMs); CTA rank c owns a contiguous slice of the n_keys
// cache positions, a whole number of 64-key tiles. The
// slice's K rows and then its V rows stream through a ring of shared-memory tiles
// of 64 consecutive cache slots of this KV head: HD/64 tensor-map TMA boxes of
// [64 slots][64 dims] with the 128-byte swizzle, so the tensor-core fragment loads
// (ldmatrix) are free of bank conflicts. Tiles are cut at the ring's wrap-around so
// their slots are contiguous. Each tile has a "full" barrier (bytes landed) and an
// "empty" barrier (all 8 warps done); warp (t mod 8) refills the stage of tile t,
// so no warp waits for another except through data. The first tiles are issued
// before the programmatic-dependent-launch wait: cache rows of earlier positions
// were written before the host synchronisation that ends every decode step, so
// they never depend on kernels still in flight.
//   phase 0  every CTA normalises and rotates its REP query heads from the raw
//            projection row; the CTA owning the newest position also normalises /
//            rotates the new K, normalises the new V and appends both to the cache
//            slot pos % cap (the tile copy of that slot is patched from shared
//            memory, never trusted);
//   phase 1  S = Q K^T with mma.sync m16n8k16 (bf16 in, fp32 accumulate; heads are
//            the M rows, zero padded to 16): warp w owns keys 8w..8w+7 of every
//            tile; s = bf16(s * scale) into shared memory; each warp reduces
//            (max, sum of exp) over its own keys; the CTA's pair is pushed into every
//            CTA of the cluster (remote stores);
//   cluster barrier; each warp merges the pushed pairs into the row's (M, L) with a
//            fixed shuffle tree (the same on every CTA) and turns its own scores into
//            p = bf16(exp(s - M) / L);
//   phase 2  O = P V with mma.sync: warp w owns head_dim columns [w HD/8, (w+1) HD/8)
//            over all keys (bf16 p is exact in rounding mode 0; mode 1 adds the
//            bf16 residual p - bf16(p) as a second product); each output element's
//            CTA partial is pushed to the CTA owning that element's slice;
//   cluster barrier; each CTA sums the pushed partials of its slice in rank order
//            (deterministic) and writes bf16.
// Only remote stores cross CTAs (no remote loads wait on latency). The cluster
// barriers are hardware barriers; every mbarrier wait is bounded.
#include "kernels.h"
#include "tma.cuh"

#include <algorithm>
#include <cfloat>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

namespace hyb {

__device__ int g_attn_wait_timeouts = 0;  // set if a stage wait gave up (never expected)

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxCluster = 16;
constexpr int kPortableCluster = 8;
constexpr int kTileKeys = 64;       // cache slots per tile (8 per warp)
constexpr int kRingBytes = 196608;  // tile bytes in flight per CTA
constexpr int kMaxStages = 8;
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

// e^x as one MUFU operation on log2(e)-scaled arguments, flushing denormal results to zero.
__device__ __forceinline__ float exp_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
    return y;
}

// (max, sum of exp relative to the max) over the lanes of one 8-lane group: `m` and `l` are
// one entry per lane (l = 0: empty); every lane of the group gets the merged pair.
__device__ __forceinline__ void merge8(float m, float l, float& M, float& L) {
    M = l > 0.f ? m : -FLT_MAX;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    L = l > 0.f ? l * exp_fast(m - M) : 0.f;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
}

// merge8 over the lanes of one 16-lane group (one entry per CTA of a cluster of <= 16).
__device__ __forceinline__ void merge16(float m, float l, float& M, float& L) {
    M = l > 0.f ? m : -FLT_MAX;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    L = l > 0.f ? l * exp_fast(m - M) : 0.f;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
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

// Normalise one head row of the raw projection (optionally rotate) into `dst`
// (floats holding bf16-rounded values). One warp; elements e = lane + 32 i.
// Not inlined: its call sites (query heads, new K, new V) share one copy of the code,
// which keeps the kernel's cold instruction fetch small (each CTA runs it once).
template <int PER>
__device__ __noinline__ void norm_rope_row(const bf16* src, const bf16* nw, const float* inv_freq, int pos, float eps,
                              bool rope, float* dst, bf16* cache_dst) {
    const int lane = threadIdx.x & 31;
    constexpr int HD = PER * 32;
    constexpr int HP = PER / 2;
    // every operand is loaded up front, so the row costs one memory latency
    float v[PER], w[PER], fr[HP];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        v[i] = bf2f(src[lane + 32 * i]);
        w[i] = nw ? bf2f(nw[lane + 32 * i]) : 1.f;
    }
#pragma unroll
    for (int i = 0; i < HP; ++i) fr[i] = rope ? inv_freq[lane + 32 * i] : 0.f;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) ss += v[i] * v[i];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const float t = rbf(v[i] * inv);
        v[i] = nw ? rbf(t * w[i]) : t;
    }
    if (rope) {
#pragma unroll
        for (int i = 0; i < HP; ++i) {
            const float f = fr[i];
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

// Shared-memory plan (bytes from a 1024-byte aligned base): tiles, barriers, floats.
struct FusedLayout {
    size_t full, empty, q_s, knew, vnew, wml, allml, recv, s_sc, total;
};

__host__ __device__ inline FusedLayout fused_layout(int hd, int rep, int chunk, int stages) {
    FusedLayout L;
    L.full = static_cast<size_t>(stages) * kTileKeys * hd * 2;
    L.empty = L.full + 8 * kMaxStages;
    size_t f = L.empty + 8 * kMaxStages;
    auto take = [&](size_t floats) {
        const size_t at = f;
        f += 4 * ((floats + 1) & ~static_cast<size_t>(1));  // keep 8-byte alignment
        return at;
    };
    const size_t E = static_cast<size_t>(rep) * hd;
    L.q_s = take(E);
    L.knew = take(hd);
    L.vnew = take(hd);
    L.wml = take(2 * static_cast<size_t>(kWarps) * rep);
    L.allml = take(2 * static_cast<size_t>(kMaxCluster) * rep);
    L.recv = take(E + kMaxCluster);
    L.s_sc = take(static_cast<size_t>(rep) * chunk);
    L.total = f;
    return L;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// Byte offset of 16-byte chunk c (8 bf16 of head_dim) of tile row r. A tile is
// HD/64 sub-tiles of [64 rows][128 bytes], each written by one TMA box with the
// 128-byte swizzle: chunk c' of row r sits at chunk c' ^ (r mod 8).
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
    return static_cast<uint32_t>((c >> 3) * (kTileKeys * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <int PER, int REP, int ROUND>
__global__ void __launch_bounds__(kThreads, 1) decode_attn_fused_kernel(const DecodeFusedParams p, int chunk,
                                                                     int stages,
                                                                     const __grid_constant__ CUtensorMap tmk,
                                                                     const __grid_constant__ CUtensorMap tmv) {
    constexpr int HD = PER * 32;
    constexpr int E = REP * HD;
    constexpr int T = kTileKeys;            // keys per tile
    constexpr int TILE = T * HD * 2;        // bytes per tile
    constexpr int SUB = HD / 64;            // 128-byte sub-tiles (TMA boxes) per tile
    constexpr int KSTEPS = HD / 16;         // MMA k-steps over head_dim
    constexpr int NTW = HD / 64;            // 8-wide output column tiles per warp in P V
    static_assert(T == 8 * kWarps, "each warp owns 8 keys of a tile");
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* smem_raw = smem_dyn + ((1024 - (smem_u32(smem_dyn) & 1023)) & 1023);  // 1024-aligned
    const FusedLayout lay = fused_layout(HD, REP, chunk, stages);
    unsigned char* tiles = smem_raw;                                  // [stages][TILE], swizzled
    float* q_s = reinterpret_cast<float*>(smem_raw + lay.q_s);      // [REP][HD]
    float* knew = reinterpret_cast<float*>(smem_raw + lay.knew);    // [HD]
    float* vnew = reinterpret_cast<float*>(smem_raw + lay.vnew);    // [HD]
    float* wml = reinterpret_cast<float*>(smem_raw + lay.wml);      // [kWarps][REP][2] per-warp (max, sum)
    float* allml = reinterpret_cast<float*>(smem_raw + lay.allml);  // [CS][REP][2] pushed by every CTA
    float* recv = reinterpret_cast<float*>(smem_raw + lay.recv);    // [CS][per_cta] pushed partials
    float* s_sc = reinterpret_cast<float*>(smem_raw + lay.s_sc);    // [REP][chunk]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;  // MMA fragment coordinates
    const int hk = blockIdx.y;
    // this CTA's sequence: the launch's own fields, or entry blockIdx.z of a batched launch
    const DecodeSeq* sq = p.seqs ? p.seqs + blockIdx.z : nullptr;
    const bf16* qkv = sq ? sq->qkv : p.qkv;
    bf16* out = sq ? sq->out : p.out;
    bf16* k_cache = sq ? sq->k_cache : p.k_cache;
    bf16* v_cache = sq ? sq->v_cache : p.v_cache;
    const int cap = sq ? sq->cap : p.cap;
    const int pos = sq ? sq->pos : p.pos;
    const int n_keys = sq ? sq->n_keys : p.n_keys;
    const CUtensorMap* map_k = sq ? &sq->tk : &tmk;
    const CUtensorMap* map_v = sq ? &sq->tv : &tmv;
    const int CS = gridDim.x;
    const uint32_t rank = cluster_rank();
    const int j0 = static_cast<int>(rank) * chunk;
    const int j1 = min(n_keys, j0 + chunk);
    const int n = max(0, j1 - j0);
    const bool owns_newest = !p.kv_ready && (j1 == n_keys) && n > 0;
    const int newest = n_keys - 1;
    const int first_pos = pos - n_keys + 1;
    // tiles: segment A = keys before the ring wraps to slot 0, segment B = the rest
    const int s_first = (first_pos + j0) % cap;
    const int lenA = min(n, cap - s_first);
    const int ntA = (lenA + T - 1) / T;
    const int nt = ntA + (n - lenA + T - 1) / T;  // K tiles (and V tiles) of this CTA
    const int items = 2 * nt;                     // item t < nt: K tile t; t >= nt: V tile t - nt
    // tile t: keys [x, y) and the first slot z of its box
    auto tile_keys = [=](int t) {
        if (t < ntA) return make_int3(j0 + t * T, min(j0 + lenA, j0 + t * T + T), s_first + t * T);
        const int jb = j0 + lenA + (t - ntA) * T;
        return make_int3(jb, min(j1, jb + T), (t - ntA) * T);
    };
    const uint32_t tiles_u32 = smem_u32(tiles);
    const uint32_t full0 = smem_u32(smem_raw + lay.full), empty0 = smem_u32(smem_raw + lay.empty);

    // The dependent kernel may launch at once (its PDL wait still waits for this grid)
    // and stream its weights meanwhile.
    pdl_launch_dependents();
    cluster_arrive_relaxed();  // matched by the wait before the first remote store
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kWarps);
        }
        mbar_init_fence();
    }
    __syncthreads();

    // Load item `it` into stage it % stages (one thread): SUB boxes of 64 slots x 64
    // dims. Rows past the tile's keys (other slots, or zero fill past cap) are never
    // used, and the newest slot, written by this kernel, is patched from registers.
    auto issue = [&](int it) {
        const bool isv = it >= nt;
        const int3 tk = tile_keys(isv ? it - nt : it);
        const int s = it % stages;
        const uint32_t fb = full0 + 8 * s;
        mbar_expect_tx(fb, TILE);
#pragma unroll
        for (int sub = 0; sub < SUB; ++sub)
            tma_load_3d_hint(tiles_u32 + s * TILE + sub * (T * 128), isv ? map_v : map_k, 64 * sub, hk, tk.z, fb,
                             l2_evict_first());
    };
    // tensor maps written to global memory by a copy: every thread that may issue a load
    // with them (the first-stage issuers below, lane 0 of each warp for refills) acquires
    // them for the TMA unit first
    if (sq && (lane == 0 || static_cast<int>(threadIdx.x) < stages)) {
        asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map_k) : "memory");
        asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map_v) : "memory");
    }
    // the first stages, one issuing thread each: K tiles now, the first V tiles after
    // phase 0 (whose loads of the projection row would otherwise queue behind them)
    const int first_v = min(stages, min(items, nt));
    if (static_cast<int>(threadIdx.x) < first_v) issue(threadIdx.x);

    pdl_wait();
    // ---- phase 0: query heads of this KV head, and the new token's K/V
    const int q_col = hk * REP * HD;
    const int k_col = p.n_heads * HD + hk * HD;
    const int v_col = p.v_from_k ? k_col : p.n_heads * HD + p.n_kv * HD + hk * HD;
    for (int r = warp; r < REP; r += kWarps - 2)
        norm_rope_row<PER>(qkv + q_col + r * HD, p.q_norm, p.inv_freq, pos, p.eps, true, q_s + r * HD,
                           nullptr);
    if (owns_newest) {
        const int slot = pos % cap;
        if (warp == kWarps - 1)
            norm_rope_row<PER>(qkv + k_col, p.k_norm, p.inv_freq, pos, p.eps, true, knew,
                               k_cache + (static_cast<size_t>(slot) * p.n_kv + hk) * HD);
        if (warp == kWarps - 2)
            norm_rope_row<PER>(qkv + v_col, nullptr, p.inv_freq, pos, p.eps, false, vnew,
                               v_cache + (static_cast<size_t>(slot) * p.n_kv + hk) * HD);
    }
    __syncthreads();
    if (static_cast<int>(threadIdx.x) >= first_v && static_cast<int>(threadIdx.x) < min(stages, items))
        issue(threadIdx.x);

    bool waits_ok = true;
    auto wait_full = [&](int it) {
        const int s = it % stages;
        if (!mbar_wait_bounded(full0 + 8 * s, static_cast<uint32_t>(it / stages) & 1u)) waits_ok = false;
        return tiles_u32 + static_cast<uint32_t>(s * TILE);
    };
    // This warp is done with item `it`; warp (it mod 8) refills the stage once all are.
    auto release = [&](int it) {
        const int s = it % stages;
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);
        if (it + stages < items && warp == it % kWarps && lane == 0) {
            if (!mbar_wait_bounded(empty0 + 8 * s, static_cast<uint32_t>(it / stages) & 1u)) waits_ok = false;
            issue(it + stages);
        }
    };
    // Overwrite columns [c0, c1) (16-byte chunks) of tile row r with `src` (floats
    // holding bf16 values): the newest slot, whose cache row this kernel just wrote.
    auto patch_row = [&](uint32_t tile, int r, const float* src, int c0, int c1) {
        for (int c = c0 + lane; c < c1; c += 32) {
            const float* v = src + 8 * c;
            uint4 w;
            w.x = pack_bf2(f2bf(v[0]), f2bf(v[1]));
            w.y = pack_bf2(f2bf(v[2]), f2bf(v[3]));
            w.z = pack_bf2(f2bf(v[4]), f2bf(v[5]));
            w.w = pack_bf2(f2bf(v[6]), f2bf(v[7]));
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(tile + tile_off(r, c)), "r"(w.x), "r"(w.y),
                         "r"(w.z), "r"(w.w)
                         : "memory");
        }
        fence_proxy_async();  // the stage is refilled by TMA later
        __syncwarp();
    };
    // key index (relative to j0) of this warp's i-th key, or -1 past its tile's keys
    auto my_key = [=](int i) {
        const int3 tk = tile_keys(i >> 3);
        const int j = tk.x + 8 * warp + (i & 7);
        return j < tk.y ? j - j0 : -1;
    };
    const int my_count = nt * 8;

    // ---- phase 1: scores S = Q K^T on tensor cores; this warp owns keys 8w..8w+7 of each tile
    {
        uint32_t qa[KSTEPS][2];  // A fragments of Q (rows = heads; rows >= REP are zero)
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
            if (g < REP) {
                const float* qr = q_s + g * HD + 16 * kk + 2 * t4;
                qa[kk][0] = pack_bf2(f2bf(qr[0]), f2bf(qr[1]));
                qa[kk][1] = pack_bf2(f2bf(qr[8]), f2bf(qr[9]));
            } else {
                qa[kk][0] = qa[kk][1] = 0u;
            }
        }
        for (int it = 0; it < nt; ++it) {
            const uint32_t tile = wait_full(it);
            const int3 tk = tile_keys(it);
            const int kb = tk.x, ke = tk.y;
            if (owns_newest && newest >= kb + 8 * warp && newest < kb + 8 * warp + 8 && newest < ke)
                patch_row(tile, newest - kb, knew, 0, HD / 8);
            // two independent accumulator chains (even and odd k-steps) halve the MMA
            // dependency chain; they are added once at the end
            float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
            const int lr = 8 * warp + (lane & 7);  // this lane's ldmatrix row
#pragma unroll
            for (int k2 = 0; k2 < KSTEPS / 2; ++k2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(tile + tile_off(lr, 4 * k2 + (lane >> 3)), b0, b1, b2, b3);
                mma_bf16_16816(acc, qa[2 * k2][0], 0u, qa[2 * k2][1], 0u, b0, b1);
                mma_bf16_16816(acc2, qa[2 * k2 + 1][0], 0u, qa[2 * k2 + 1][1], 0u, b2, b3);
            }
            acc[0] += acc2[0];
            acc[1] += acc2[1];
            if (g < REP) {
                const int j = kb + 8 * warp + 2 * t4;
                if (j < ke) s_sc[g * chunk + (j - j0)] = score_round(acc[0], p.scale, p.softcap, ROUND);
                if (j + 1 < ke) s_sc[g * chunk + (j + 1 - j0)] = score_round(acc[1], p.scale, p.softcap, ROUND);
            }
            release(it);
        }
    }
    // ---- this warp's (max, sum of exp) per head over its own keys, every head in the
    // same passes (independent shuffle chains)
    {
        float m[REP], l[REP];
#pragma unroll
        for (int h = 0; h < REP; ++h) {
            m[h] = -FLT_MAX;
            l[h] = 0.f;
        }
        for (int i = lane; i < my_count; i += 32) {
            const int k = my_key(i);
            if (k >= 0) {
#pragma unroll
                for (int h = 0; h < REP; ++h) m[h] = fmaxf(m[h], s_sc[h * chunk + k]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int h = 0; h < REP; ++h) m[h] = fmaxf(m[h], __shfl_xor_sync(0xffffffffu, m[h], o));
        for (int i = lane; i < my_count; i += 32) {
            const int k = my_key(i);
            if (k >= 0) {
#pragma unroll
                for (int h = 0; h < REP; ++h) l[h] += exp_fast(s_sc[h * chunk + k] - m[h]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int h = 0; h < REP; ++h) l[h] += __shfl_xor_sync(0xffffffffu, l[h], o);
        if (lane == 0) {
#pragma unroll
            for (int h = 0; h < REP; ++h) {
                wml[(warp * REP + h) * 2] = m[h];
                wml[(warp * REP + h) * 2 + 1] = l[h];
            }
        }
    }
    __syncthreads();
    // every CTA of the cluster has started: its shared memory may now be written
    cluster_wait();
    // warp h merges head h's (max, sum) over the 8 warps (lanes 0..7, shuffle tree) and
    // lanes c < CS push the CTA's pair into CTA c
    if (warp < REP) {
        const int h = warp, w = lane & 7;
        float M, L;
        merge8(wml[(w * REP + h) * 2], wml[(w * REP + h) * 2 + 1], M, L);
        if (lane < CS) dsmem_st2(dsmem_addr(&allml[(rank * REP + h) * 2], lane), M, L);
    }
    cluster_sync();
    // ---- row statistics (lane h < REP), then p in place over this warp's keys
    {
        // heads in pairs, one per 16-lane half: lane c (< CS) of a half holds CTA c's pair
        // for its head, and the half's shuffle tree merges them
        float Mh[REP], iLh[REP];
#pragma unroll
        for (int h0 = 0; h0 < REP; h0 += 2) {
            const int hh = h0 + (lane >> 4);
            const int c = lane & 15;
            const bool has = c < CS && hh < REP;
            float M, L;
            merge16(has ? allml[(c * REP + hh) * 2] : -FLT_MAX, has ? allml[(c * REP + hh) * 2 + 1] : 0.f, M, L);
            const float iL = 1.0f / L;
            Mh[h0] = __shfl_sync(0xffffffffu, M, 0);
            iLh[h0] = __shfl_sync(0xffffffffu, iL, 0);
            if (h0 + 1 < REP) {
                Mh[h0 + 1] = __shfl_sync(0xffffffffu, M, 16);
                iLh[h0 + 1] = __shfl_sync(0xffffffffu, iL, 16);
            }
        }
        for (int i = lane; i < my_count; i += 32) {
            const int k = my_key(i);
            if (k >= 0) {
#pragma unroll
                for (int h = 0; h < REP; ++h) {
                    const float e = exp_fast(s_sc[h * chunk + k] - Mh[h]) * iLh[h];
                    s_sc[h * chunk + k] = (ROUND == 0) ? rbf(e) : e;
                }
            }
        }
    }
    __syncthreads();  // P V reads every warp's probabilities
    // ---- phase 2: O = P V on tensor cores; this warp owns head_dim columns [w HD/8, (w+1) HD/8)
    float o[NTW][4];
#pragma unroll
    for (int nn = 0; nn < NTW; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
    for (int it = nt; it < items; ++it) {
        const uint32_t tile = wait_full(it);
        const int3 tk = tile_keys(it - nt);
        const int kb = tk.x, ke = tk.y;
        if (owns_newest && newest >= kb && newest < ke)
            patch_row(tile, newest - kb, vnew, warp * NTW, warp * NTW + NTW);
#pragma unroll
        for (int kk = 0; kk < T / 16; ++kk) {
            // A fragment: p[head g][keys kb + 16 kk + {2t, 2t+1, 2t+8, 2t+9}], zero past the tile's keys
            float pv[4] = {0.f, 0.f, 0.f, 0.f};
            if (g < REP) {
                const int jj = kb + 16 * kk + 2 * t4;
                const float* pr = s_sc + g * chunk - j0;
                if (jj < ke) pv[0] = pr[jj];
                if (jj + 1 < ke) pv[1] = pr[jj + 1];
                if (jj + 8 < ke) pv[2] = pr[jj + 8];
                if (jj + 9 < ke) pv[3] = pr[jj + 9];
            }
            const bf16 h0 = f2bf(pv[0]), h1 = f2bf(pv[1]), h2 = f2bf(pv[2]), h3 = f2bf(pv[3]);
            const uint32_t a0 = pack_bf2(h0, h1), a2 = pack_bf2(h2, h3);
            uint32_t l0 = 0u, l2 = 0u;  // rounding mode 1: fp32 p = hi + lo in two bf16 products
            if (ROUND != 0) {
                l0 = pack_bf2(f2bf(pv[0] - bf2f(h0)), f2bf(pv[1] - bf2f(h1)));
                l2 = pack_bf2(f2bf(pv[2] - bf2f(h2)), f2bf(pv[3] - bf2f(h3)));
            }
            const int lr = 16 * kk + 8 * ((lane >> 3) & 1) + (lane & 7);  // this lane's ldmatrix row (key)
            if constexpr (NTW == 1) {
                uint32_t b0, b1;
                ldsm_x2_t(tile + tile_off(lr, warp), b0, b1);
                mma_bf16_16816(o[0], a0, 0u, a2, 0u, b0, b1);
                if (ROUND != 0) mma_bf16_16816(o[0], l0, 0u, l2, 0u, b0, b1);
            } else {
#pragma unroll
                for (int nn = 0; nn < NTW; nn += 2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(tile + tile_off(lr, warp * NTW + nn + (lane >> 4)), b0, b1, b2, b3);
                    mma_bf16_16816(o[nn], a0, 0u, a2, 0u, b0, b1);
                    mma_bf16_16816(o[nn + 1], a0, 0u, a2, 0u, b2, b3);
                    if (ROUND != 0) {
                        mma_bf16_16816(o[nn], l0, 0u, l2, 0u, b0, b1);
                        mma_bf16_16816(o[nn + 1], l0, 0u, l2, 0u, b2, b3);
                    }
                }
            }
        }
        release(it);
    }
    // ---- push each output element's CTA partial to the CTA owning its slice
    const int per_cta = (E + CS - 1) / CS;
    if (g < REP) {
#pragma unroll
        for (int nn = 0; nn < NTW; ++nn) {
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int i = g * HD + (warp * NTW + nn) * 8 + 2 * t4 + q;
                const int owner = i / per_cta;
                dsmem_st(dsmem_addr(&recv[rank * per_cta + (i - owner * per_cta)], owner), o[nn][q]);
            }
        }
    }
    cluster_sync();
    // ---- this CTA's slice, summed in rank order
    const int e0 = static_cast<int>(rank) * per_cta, e1 = min(E, e0 + per_cta);
    for (int i = e0 + static_cast<int>(threadIdx.x); i < e1; i += kThreads) {
        float v = 0.f;
        for (int c = 0; c < CS; ++c) v += recv[c * per_cta + (i - e0)];
        out[static_cast<size_t>(hk * REP) * HD + i] = f2bf(v);
    }
    if (__syncthreads_or(!waits_ok) && threadIdx.x == 0) {
        atomicAdd(&g_attn_wait_timeouts, 1);
        // copies that never signalled may still land: wait (bounded) before the CTA exits
        for (int s = 0; s < stages && s < items; ++s)
            mbar_wait_bounded(full0 + 8 * s, static_cast<uint32_t>((items - 1 - s) / stages) & 1u);
    }
}

struct FusedPlan {
    int cs = 0, chunk = 0, stages = 0;
    size_t smem = 0;
};

// `units` = independent (KV head, sequence) pairs of the launch, `cs_cap` the largest
// cluster allowed. While the launch has fewer pairs than SMs, a cluster splits a pair's
// keys over up to SMs / units CTAs in whole 64-key tiles (the most tiles on any CTA as
// low as the SMs allow) and each CTA keeps up to 192 KB of tiles in flight; a launch with
// a pair or more per SM runs one CTA per pair with 128 KB in flight, leaving room for
// more resident CTAs. A plan whose scores do not fit in shared memory takes more CTAs per
// cluster.
FusedPlan plan_fused(int hd, int rep, int n_keys, int units, int cs_cap) {
    const int sms = num_sms();
    const int tiles = (n_keys + kTileKeys - 1) / kTileKeys;
    const int want = std::max(1, std::min(cs_cap, sms / std::max(units, 1)));
    const int ring = units < sms ? kRingBytes : 131072;
    const int tile = kTileKeys * hd * 2;
    for (int c = want; c <= cs_cap; ++c) {
        FusedPlan f;
        f.chunk = (tiles + c - 1) / c * kTileKeys;
        f.cs = (n_keys + f.chunk - 1) / f.chunk;
        // +1 tile for a possible split at the ring wrap
        const int items = 2 * (f.chunk / kTileKeys + 1);
        for (int s = std::min({kMaxStages, items, ring / tile}); s >= 1; --s) {
            f.stages = s;
            f.smem = fused_layout(hd, rep, f.chunk, s).total + 1024;  // + alignment slack
            if (f.smem <= kSmemLimit) return f;
        }
    }
    return FusedPlan{};
}

// Clusters of `cs` CTAs of `kern` with `smem` bytes each that the device keeps resident
// at once (cached per device, cluster size and shared memory).
template <typename K>
int resident_clusters(K kern, int cs, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, size_t>, int> cache;
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_tuple(dev, cs, smem);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
    }
    cache[key] = n;
    return n;
}

template <int PER, int REP, int ROUND>
void launch_fused_t(const DecodeFusedParams& p, cudaStream_t stream, bool pdl) {
    const int units = p.n_kv * (p.seqs ? p.n_seq : 1);
    auto kern = decode_attn_fused_kernel<PER, REP, ROUND>;
    static int attr_dev = -1;
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        HYB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit)));
        HYB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        attr_dev = dev;
    }
    // clusters above the portable 8 CTAs only where all of the launch's clusters fit at
    // once: the largest such size (each smaller cap may give fewer tiles per CTA than 8)
    FusedPlan f = plan_fused(PER * 32, REP, p.n_keys, units, kMaxCluster);
    while (f.stages != 0 && f.cs > kPortableCluster && resident_clusters(kern, f.cs, f.smem) < units)
        f = plan_fused(PER * 32, REP, p.n_keys, units, f.cs - 1);
    if (f.stages == 0) throw ArgError("decode attention: too many keys for the shared-memory plan");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(f.cs, p.n_kv, p.seqs ? p.n_seq : 1);
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
    CUtensorMap tk{}, tv{};  // a batched launch reads every sequence's maps from p.seqs
    if (!p.seqs) {
        if (p.tmap_k) tk = *p.tmap_k;
        else encode_kv_tensor_map(&tk, p.k_cache, p.cap, p.n_kv, p.hd);
        if (p.tmap_v) tv = *p.tmap_v;
        else encode_kv_tensor_map(&tv, p.v_cache, p.cap, p.n_kv, p.hd);
    }
    HYB_CUDA(cudaLaunchKernelEx(&cfg, kern, p, f.chunk, f.stages, tk, tv));
}

template <int PER>
void launch_fused_rep(const DecodeFusedParams& p, cudaStream_t stream, bool pdl) {
    switch (p.n_heads / p.n_kv) {
        case 1:
            if (p.rounding == 0) launch_fused_t<PER, 1, 0>(p, stream, pdl);
            else launch_fused_t<PER, 1, 1>(p, stream, pdl);
            break;
        case 2:
            if (p.rounding == 0) launch_fused_t<PER, 2, 0>(p, stream, pdl);
            else launch_fused_t<PER, 2, 1>(p, stream, pdl);
            break;
        case 4:
            if (p.rounding == 0) launch_fused_t<PER, 4, 0>(p, stream, pdl);
            else launch_fused_t<PER, 4, 1>(p, stream, pdl);
            break;
        case 8:
            if (p.rounding == 0) launch_fused_t<PER, 8, 0>(p, stream, pdl);
            else launch_fused_t<PER, 8, 1>(p, stream, pdl);
            break;
        default: throw ArgError("decode attention: GQA group must be 1, 2, 4 or 8");
    }
}

}  // namespace

void encode_kv_tensor_map(CUtensorMap* map, const bf16* cache, int cap, int n_kv, int hd) {
    if (cap <= 0 || n_kv <= 0 || (hd != 64 && hd != 128 && hd != 256))
        throw ArgError("decode attention: bad K/V cache for a tensor map");
    const uint64_t dims[3] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(n_kv), static_cast<uint64_t>(cap)};
    const uint64_t strides[2] = {static_cast<uint64_t>(hd) * 2, static_cast<uint64_t>(n_kv) * hd * 2};
    const uint32_t box[3] = {64, 1, static_cast<uint32_t>(kTileKeys)};  // 128-byte rows, swizzled
    encode_tma(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, cache, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool decode_attn_fused_fits(int n_heads, int n_kv, int hd, int n_keys) {
    if (n_kv <= 0 || n_heads % n_kv != 0 || (hd != 64 && hd != 128 && hd != 256) || n_keys <= 0) return false;
    const int rep = n_heads / n_kv;
    if (rep != 1 && rep != 2 && rep != 4 && rep != 8) return false;
    // the portable plan always launches, so it decides whether the fused kernel applies
    return plan_fused(hd, rep, n_keys, n_kv, kPortableCluster).stages > 0;
}

void launch_decode_attn_fused(const DecodeFusedParams& p, cudaStream_t stream, bool pdl) {
    if (p.kv_ready && pdl) throw ArgError("decode attention: kv_ready launches cannot use PDL");
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

void launch_decode_attn_fused_batch(const DecodeFusedParams& p, int n_keys_max, cudaStream_t stream, bool pdl) {
    if (!p.seqs || p.n_seq < 1 || p.n_seq > 65535 || (reinterpret_cast<uintptr_t>(p.seqs) & 63))
        throw ArgError("decode attention batch: sequences must be a 64-byte aligned device array");
    if (n_keys_max <= 0 || p.n_kv <= 0 || p.n_heads % p.n_kv != 0)
        throw ArgError("decode attention batch: bad shape");
    if ((p.n_heads / p.n_kv) * p.hd > 1024) throw ArgError("decode attention: GQA group x head_dim > 1024");
    // cache tiles are requested before the dependency wait: appended K/V must be complete
    if (p.kv_ready && pdl) throw ArgError("decode attention batch: kv_ready launches cannot use PDL");
    DecodeFusedParams q = p;
    q.n_keys = n_keys_max;  // the shared-memory plan covers the longest sequence
    switch (p.hd) {
        case 64: launch_fused_rep<2>(q, stream, pdl); break;
        case 128: launch_fused_rep<4>(q, stream, pdl); break;
        case 256: launch_fused_rep<8>(q, stream, pdl); break;
        default: throw ArgError("decode attention: head_dim must be 64, 128 or 256");
    }
}

int64_t read_attn_wait_timeouts() {
    int a = 0;
    HYB_CUDA(cudaMemcpyFromSymbol(&a, g_attn_wait_timeouts, sizeof(int)));
    return a;
}

}  // namespace hyb
