// Batch-1 affine Q4/g64 qmv over the engine's packed resident weight layout,
// streamed with TMA bulk copies (cp.async.bulk + mbarrier) into per-warp
// shared-memory rings.
//
// Same mathematics and MMA formulation as qmv.cu (codes as bf16 128 + q on the
// A side, per-unit group-masked activations on the B side, per-group
// scale/bias fold in fp32); only the data movement differs.
//
// Packed layout (built once at load by launch_qmv_pack from the MLX layout
// [N, K/8] u32 + [N, K/64] bf16 scales/biases):
//   rows are grouped in 16-row blocks (zero padded), K in 512-wide units of
//   8 groups (the last unit may hold fewer). For block rb and unit u the item is
//   one contiguous run of nv * 144 bytes, nv = 8 * ceil(gc / 2) valid lanes:
//     chunk c (0..7) of every valid lane, then one 16-byte scale/bias record per
//     lane. Lane (g, t) owns rows g and g + 8 and groups 2t, 2t + 1 of the unit;
//     chunk c = (row h = c / 4, 16-byte piece c % 4 of its 64-byte segment).
//     The record holds bf16 {sA(g), sB(g), sA(g+8), sB(g+8), bA(g), bB(g),
//     bA(g+8), bB(g+8)}. Lane rank = g * tv + t with tv = ceil(gc / 2).
//   A warp's reads of one chunk index are 32 consecutive 16-byte words, so the
//   shared-memory reads are conflict-free, and each item is a single bulk copy.
#include "kernels.h"
#include "qmv_pack.cuh"
#include "tma.cuh"

#include <algorithm>
#include <type_traits>

namespace hyb {

__device__ int g_qmv_wait_timeouts = 0;  // set if an mbarrier wait gave up (never expected)

namespace {

// One CTA of 16 warps per SM (<= 128 registers, <= ~184 KB shared memory): the work
// splits per SM, so row-block counts that do not divide evenly cost at most one group
// per SM (two 8-warp CTAs per SM left some SMs with both CTAs busy and others with one),
// and the norm prologue runs once per SM.
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 2;
constexpr int kCtasPerSm = 1;
constexpr int kMaxPrologueK = 8192; // norm prologues hold K/8 16-byte chunks in registers

// Bounded wait on an mbarrier phase: gives up (and records it) instead of hanging.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
    if (mbar_wait_bounded(bar, phase)) return true;
    atomicAdd(&g_qmv_wait_timeouts, 1);
    return false;
}

// Sum over the CTA in a fixed order (warp trees, then the warps' partials in warp order),
// so every CTA gets the same bits. `slot` (0 or 1) picks the partials' buffer: each slot
// is used once per launch, so one barrier suffices.
__device__ __forceinline__ float block_sum(float v, float* tmp, int slot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) tmp[slot * kWarps + warp] = v;
    __syncthreads();
    float r = (lane < kWarps) ? tmp[slot * kWarps + lane] : 0.f;
    return warp_sum(r);
}

// Operands of a norm prologue that do not depend on earlier kernels (norm weights, the
// post-norm weights and the layer scalar), loaded before the dependent-launch wait.
constexpr int kMaxPrologueChunks = (kMaxPrologueK / 8 + kThreads - 1) / kThreads;
struct PrologueWeights {
    uint4 nw[kMaxPrologueChunks], pw[kMaxPrologueChunks];
    float scalar = 1.f;
};

__device__ __forceinline__ PrologueWeights load_prologue_weights(const QmvParams& p) {
    PrologueWeights w;
    const int nch = p.K / 8;
    const uint64_t keep = l2_evict_last();  // norm weights: re-read every token
    const bool resid = p.prologue == QmvPrologue::kResidNorm;
#pragma unroll
    for (int c = 0; c < kMaxPrologueChunks; ++c) {
        const int j = static_cast<int>(threadIdx.x) + c * kThreads;
        const uint4 z = make_uint4(0, 0, 0, 0);
        w.nw[c] = j < nch ? ld_v4_hint(reinterpret_cast<const uint4*>(p.norm_w) + j, keep) : z;
        w.pw[c] = (resid && j < nch) ? ld_v4_hint(reinterpret_cast<const uint4*>(p.post_w) + j, keep) : z;
    }
    if (resid && p.scalar) w.scalar = bf2f(p.scalar[0]);
    return w;
}

// ---- fused tensor-parallel all-reduce (QmvTpFuse)
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const void* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(void* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Producer: rows 2k and 2k + 1 (row 2k + 1 past N is zero) as one flagged word into slot
// (set, me) of every rank.
__device__ __forceinline__ void ar_store_pair(const QmvParams& p, int row2k, bf16 a, bf16 b) {
    const unsigned long long w =
        (static_cast<unsigned long long>(p.ar.epoch) << 32) | pack_bf2(a, row2k + 1 < p.N ? b : f2bf(0.f));
    const size_t off =
        p.ar.ll_off + ((static_cast<size_t>(p.ar.set) * p.ar.T + p.ar.me) * (p.ar.max_count / 2) + row2k / 2) * 8;
    for (int r = 0; r < p.ar.T; ++r) st_relaxed_sys_u64(p.ar.peer[r] + off, w);
}

// Consumer: chunk j (8 elements = 4 words per source) of the all-reduced vector, each word
// awaited (bounded) until it carries this all-reduce's epoch, summed over sources in rank
// order in fp32 and rounded to bf16.
__device__ __forceinline__ uint4 ar_chunk(const QmvParams& p, int j) {
    const unsigned char* mine = p.ar.peer[p.ar.me];
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    for (int src = 0; src < p.ar.T; ++src) {
        const unsigned char* slot =
            mine + p.ar.ll_off + (static_cast<size_t>(p.ar.set) * p.ar.T + src) * (p.ar.max_count / 2) * 8;
        // the source's four words as independent loads (one round trip), then each
        // re-read only while it does not yet carry this all-reduce's epoch
        unsigned long long ws[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) ws[q] = ld_relaxed_sys_u64(slot + (static_cast<size_t>(4 * j + q)) * 8);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const void* wp = slot + (static_cast<size_t>(4 * j + q)) * 8;
            unsigned long long w = ws[q];
            for (int it = 0; static_cast<unsigned>(w >> 32) != p.ar.epoch; ++it) {
                if (it >= (1 << 22)) {
                    ok = false;
                    break;
                }
                if (it > 64) __nanosleep(32);
                w = ld_relaxed_sys_u64(wp);
            }
            const uint32_t d = static_cast<uint32_t>(w);
            a[2 * q] += __uint_as_float(d << 16);
            a[2 * q + 1] += __uint_as_float(d & 0xFFFF0000u);
        }
    }
    if (!ok) atomicAdd(reinterpret_cast<int*>(p.ar.peer[p.ar.me] + p.ar.err_off), 1);
    uint4 o;
    o.x = pack_bf2(f2bf(a[0]), f2bf(a[1]));
    o.y = pack_bf2(f2bf(a[2]), f2bf(a[3]));
    o.z = pack_bf2(f2bf(a[4]), f2bf(a[5]));
    o.w = pack_bf2(f2bf(a[6]), f2bf(a[7]));
    return o;
}

// The input vector into shared memory: x (or its norm prologue) as the permuted
// bf16 pairs the MMA B fragments read, and the per-group sums of x.
// `after_loads` runs once every load of x (and resid) is issued: the kernel issues the rest
// of its first weight stages there, so those loads do not queue behind the bulk copies.
template <bool AR, typename AfterLoads>
__device__ __forceinline__ void stage_input(const QmvParams& p, const PrologueWeights& pw, uint32_t* xp, float* xsum,
                                            float* tmp, AfterLoads after_loads) {
    auto ld = [](const uint4* a) { return *a; };
    const int K = p.K;
    if (p.prologue == QmvPrologue::kNone) {
        // 16-byte chunk j of x holds x[8j .. 8j+7], which is exactly the four permuted
        // pairs xp[4j .. 4j+3] = (x[8j+p], x[8j+p+4]), p < 4. The 8 chunks of a group sit
        // in 8 consecutive lanes, which reduce its sum. Every thread issues all its loads
        // of a round (up to kRound chunks: K <= 16384 in one round trip) before using any.
        constexpr int kRound = 4;
        const int nch = K / 8;
        const uint4* xv = reinterpret_cast<const uint4*>(p.x);
        for (int base = 0; base < nch; base += kRound * kThreads) {
            uint4 v[kRound];
#pragma unroll
            for (int c = 0; c < kRound; ++c) {
                const int j = base + static_cast<int>(threadIdx.x) + c * kThreads;
                v[c] = j < nch ? ld(xv + j) : make_uint4(0, 0, 0, 0);
            }
            if (base == 0) after_loads();
#pragma unroll
            for (int c = 0; c < kRound; ++c) {
                if (base + c * kThreads >= nch) break;  // block-uniform
                const int j = base + static_cast<int>(threadIdx.x) + c * kThreads;
                const uint32_t w[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
                float part = 0.f;
#pragma unroll
                for (int q = 0; q < 4; ++q) part += __uint_as_float(w[q] << 16) + __uint_as_float(w[q] & 0xFFFF0000u);
                if (j < nch) {
                    // pairs: p = 0: (w0.lo, w2.lo), p = 1: (w0.hi, w2.hi), p = 2: (w1.lo, w3.lo), p = 3: (w1.hi, w3.hi)
                    uint4 o;
                    o.x = (w[0] & 0xFFFFu) | (w[2] << 16);
                    o.y = (w[0] >> 16) | (w[2] & 0xFFFF0000u);
                    o.z = (w[1] & 0xFFFFu) | (w[3] << 16);
                    o.w = (w[1] >> 16) | (w[3] & 0xFFFF0000u);
                    *reinterpret_cast<uint4*>(xp + 4 * j) = o;
                }
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                part += __shfl_xor_sync(0xffffffffu, part, 4);
                if (j < nch && (j & 7) == 0) xsum[j >> 3] = part;
            }
        }
    } else {
        // Norm prologues in one round trip: every thread loads its 16-byte chunks of x
        // (and resid) with independent vector loads into registers (the weights came in
        // before the dependent-launch wait), then the reductions and the permuted-pair
        // writes work from registers. Chunk c of a thread exists only if K > 4096 c
        // (block-uniform, so the branch costs nothing).
        constexpr int kMaxC = kMaxPrologueChunks;
        const int nch = K / 8;
        const int nc = (nch + kThreads - 1) / kThreads;
        const uint4* x4 = reinterpret_cast<const uint4*>(p.x);
        const bool resid = p.prologue == QmvPrologue::kResidNorm;
        const bool ar = AR && p.ar_mode == 2;
        uint4 xv[kMaxC], rv[kMaxC];
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) {
            const int j = static_cast<int>(threadIdx.x) + c * kThreads;
            const uint4 z = make_uint4(0, 0, 0, 0);
            xv[c] = rv[c] = z;
            if (c < nc && j < nch) {
                xv[c] = ar ? ar_chunk(p, j) : ld(x4 + j);
                if (resid) rv[c] = ld(reinterpret_cast<const uint4*>(p.resid) + j);
            }
        }
        after_loads();
        auto lo = [](uint32_t w) { return __uint_as_float(w << 16); };
        auto hi = [](uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); };
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) {
            if (c >= nc) break;
            const uint32_t w[4] = {xv[c].x, xv[c].y, xv[c].z, xv[c].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) ss += lo(w[q]) * lo(w[q]) + hi(w[q]) * hi(w[q]);
        }
        float inv = 1.0f / sqrtf(block_sum(ss, tmp, 0) / static_cast<float>(K) + p.eps);
        if (resid) {
            const float sc = pw.scalar;
            float ss2 = 0.f;
#pragma unroll
            for (int c = 0; c < kMaxC; ++c) {
                if (c >= nc) break;
                uint32_t w[4] = {xv[c].x, xv[c].y, xv[c].z, xv[c].w};
                const uint32_t r[4] = {rv[c].x, rv[c].y, rv[c].z, rv[c].w};
                const uint32_t pw4[4] = {pw.pw[c].x, pw.pw[c].y, pw.pw[c].z, pw.pw[c].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float h0 = rbf(lo(r[q]) + rbf(rbf(lo(w[q]) * inv) * lo(pw4[q])));
                    float h1 = rbf(hi(r[q]) + rbf(rbf(hi(w[q]) * inv) * hi(pw4[q])));
                    if (p.scalar) {
                        h0 = rbf(h0 * sc);
                        h1 = rbf(h1 * sc);
                    }
                    ss2 += h0 * h0 + h1 * h1;
                    w[q] = pack_bf2(f2bf(h0), f2bf(h1));
                }
                xv[c] = make_uint4(w[0], w[1], w[2], w[3]);
                const int j = static_cast<int>(threadIdx.x) + c * kThreads;
                if (blockIdx.x == 0 && p.h_out && j < nch) reinterpret_cast<uint4*>(p.h_out)[j] = xv[c];
            }
            inv = 1.0f / sqrtf(block_sum(ss2, tmp, 1) / static_cast<float>(K) + p.eps);
        }
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) {
            if (c >= nc) break;
            const int j = static_cast<int>(threadIdx.x) + c * kThreads;
            const uint32_t w[4] = {xv[c].x, xv[c].y, xv[c].z, xv[c].w};
            const uint32_t nw[4] = {pw.nw[c].x, pw.nw[c].y, pw.nw[c].z, pw.nw[c].w};
            uint32_t o[4];
            float part = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float y0 = rbf(rbf(lo(w[q]) * inv) * lo(nw[q]));
                const float y1 = rbf(rbf(hi(w[q]) * inv) * hi(nw[q]));
                part += y0 + y1;
                o[q] = pack_bf2(f2bf(y0), f2bf(y1));
            }
            if (j < nch) {
                uint4 pr;  // permuted pairs (x[8j+p], x[8j+p+4])
                pr.x = (o[0] & 0xFFFFu) | (o[2] << 16);
                pr.y = (o[0] >> 16) | (o[2] & 0xFFFF0000u);
                pr.z = (o[1] & 0xFFFFu) | (o[3] << 16);
                pr.w = (o[1] >> 16) | (o[3] & 0xFFFF0000u);
                *reinterpret_cast<uint4*>(xp + 4 * j) = pr;
            }
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            part += __shfl_xor_sync(0xffffffffu, part, 4);
            if (j < nch && (j & 7) == 0) xsum[j >> 3] = part;
        }
    }
}

// One 16-row x 512-code item from shared memory `st`: the lane's rows g and g + 8
// accumulate into acc0 / acc1 (codes as bf16 128 + q times the permuted activation
// pairs on the tensor cores, then the per-group scale and bias fold in fp32). Full
// units (8 groups: every lane valid) skip the per-lane validity selects; only the
// last unit of a row can be partial.
// `after_reads` runs once the item's bytes are in registers: its ring stage is free then.
template <bool FULL, typename AfterReads>
__device__ __forceinline__ void qmv_item(const unsigned char* st, const uint32_t* xp, const uint32_t* zero_page,
                                         const float* xsum, const PackGeo& pg, int unit, int g, int t, float& acc0,
                                         float& acc1, AfterReads after_reads) {
    const int tv = FULL ? 4 : (pg.gc_last + 1) / 2;
    const int nv = 8 * tv;
    const bool valid = FULL || t < tv;
    const int rank = g * tv + t;
    uint4 wv[8];
#pragma unroll
    for (int c = 0; c < 8; ++c)
        wv[c] = valid ? *reinterpret_cast<const uint4*>(st + (c * nv + rank) * 16) : make_uint4(0, 0, 0, 0);
    const uint4 sb =
        valid ? *reinterpret_cast<const uint4*>(st + (8 * nv + rank) * 16) : make_uint4(0, 0, 0, 0);
    after_reads();
    const int gA = unit * 8 + 2 * t;
    const uint32_t* src0 = (g == 2 * t && (FULL || gA < pg.G)) ? xp + gA * 32 : zero_page;
    const uint32_t* src1 = (g == 2 * t + 1 && (FULL || gA + 1 < pg.G)) ? xp + (gA + 1) * 32 : zero_page;
    // four independent accumulator chains (one per nibble pair) shorten the
    // MMA dependency chain to 8
    float d[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint4 b0v = *reinterpret_cast<const uint4*>(src0 + 4 * i);
        const uint4 b1v = *reinterpret_cast<const uint4*>(src1 + 4 * i);
        const uint32_t b0s[4] = {b0v.x, b0v.y, b0v.z, b0v.w};
        const uint32_t b1s[4] = {b1v.x, b1v.y, b1v.z, b1v.w};
        // word i of group A (chunks 0,1 row g; 4,5 row g+8) and group B (2,3 / 6,7)
        const uint4 ra0 = wv[i >> 2], ra1 = wv[4 + (i >> 2)];
        const uint4 rb0 = wv[2 + (i >> 2)], rb1 = wv[6 + (i >> 2)];
        const int cc = i & 3;
        const uint32_t xa0 = cc == 0 ? ra0.x : cc == 1 ? ra0.y : cc == 2 ? ra0.z : ra0.w;
        const uint32_t xa1 = cc == 0 ? ra1.x : cc == 1 ? ra1.y : cc == 2 ? ra1.z : ra1.w;
        const uint32_t xb0 = cc == 0 ? rb0.x : cc == 1 ? rb0.y : cc == 2 ? rb0.z : rb0.w;
        const uint32_t xb1 = cc == 0 ? rb1.x : cc == 1 ? rb1.y : cc == 2 ? rb1.z : rb1.w;
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
            const uint32_t a0 = lop3_and_or(xa0 >> (4 * pp), 0x000F000Fu, 0x43004300u);
            const uint32_t a1 = lop3_and_or(xa1 >> (4 * pp), 0x000F000Fu, 0x43004300u);
            const uint32_t a2 = lop3_and_or(xb0 >> (4 * pp), 0x000F000Fu, 0x43004300u);
            const uint32_t a3 = lop3_and_or(xb1 >> (4 * pp), 0x000F000Fu, 0x43004300u);
            mma_bf16_16816(d[pp], a0, a1, a2, a3, b0s[pp], b1s[pp]);
        }
    }
    float d0[4], d1[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        d0[c] = d[0][c] + d[2][c];
        d1[c] = d[1][c] + d[3][c];
    }
    const float xsA = (FULL || gA < pg.G) ? xsum[gA] : 0.f;
    const float xsB = (FULL || gA + 1 < pg.G) ? xsum[gA + 1] : 0.f;
    // record: {sA(g), sB(g), sA(g+8), sB(g+8), bA(g), bB(g), bA(g+8), bB(g+8)}
    const float sA0 = __uint_as_float(sb.x << 16), sB0 = __uint_as_float(sb.x & 0xFFFF0000u);
    const float sA1 = __uint_as_float(sb.y << 16), sB1 = __uint_as_float(sb.y & 0xFFFF0000u);
    const float bA0 = __uint_as_float(sb.z << 16), bB0 = __uint_as_float(sb.z & 0xFFFF0000u);
    const float bA1 = __uint_as_float(sb.w << 16), bB1 = __uint_as_float(sb.w & 0xFFFF0000u);
    acc0 = fmaf(sA0, d0[0] + d1[0], acc0);
    acc0 = fmaf(sB0, d0[1] + d1[1], acc0);
    acc0 = fmaf(fmaf(-128.f, sA0, bA0), xsA, acc0);
    acc0 = fmaf(fmaf(-128.f, sB0, bB0), xsB, acc0);
    acc1 = fmaf(sA1, d0[2] + d1[2], acc1);
    acc1 = fmaf(sB1, d0[3] + d1[3], acc1);
    acc1 = fmaf(fmaf(-128.f, sA1, bA1), xsA, acc1);
    acc1 = fmaf(fmaf(-128.f, sB1, bB1), xsB, acc1);
}

// GEGLU: the interleaved gate/up matrix alternates 16-row gate blocks (even) and the
// matching up blocks (odd); a CTA processes them as one pair so the epilogue can
// combine them. BG = row blocks per work group.

// Work split: the CTA's 8 warps form teams of `team` warps (1, 2, 4 or 8). A team
// owns whole work groups (one 16-row block, or a gate/up block pair for GEGLU) and
// splits their K units among its warps; only the team synchronises, on its own
// named barrier, to sum the warps' partials. With team = 1 warps run fully
// independently, which keeps their bulk-copy rings streaming on large N.
// AR: the fused tensor-parallel all-reduce paths are compiled in (tensor-parallel launches only).
template <bool GEGLU, bool AR>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) qmv_packed_kernel(const QmvParams p, int team) {
    constexpr int BG = GEGLU ? 2 : 1;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const PackGeo pg = pack_geo(p.K, p.N);
    const unsigned char* packed = static_cast<const unsigned char*>(p.packed);

    // shared memory: [rings kWarps x kStages x 4608][mbar kWarps x kStages][xp K/2 u32][zero 32]
    //                [xsum G][red 2 x kWarps x 16][pair kWarps x 32][tmp 32]
    unsigned char* ring = smem_raw;
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kWarps * kStages * kItemMax);
    uint32_t* xp = reinterpret_cast<uint32_t*>(bars + kWarps * kStages);
    uint32_t* zero_page = xp + p.K / 2;
    float* xsum = reinterpret_cast<float*>(zero_page + 32);
    float* red = xsum + ((pg.G + 3) & ~3);
    float* pairbuf = red + 2 * kWarps * 16;
    float* tmp = pairbuf + kWarps * 32;

    unsigned char* my_ring = ring + warp * kStages * kItemMax;
    const uint32_t my_bar0 = smem_u32(bars + warp * kStages);

    const int W = team;
    const int tw = warp / W, wt = warp % W;  // team within the CTA, warp within the team
    // Groups are dealt round-robin over the CTAs (one per SM), so every SM gets the same
    // count within one: CTA b owns groups b, b + grid, b + 2 grid, ..., and its team tw
    // takes every tpc-th of them starting at the tw-th.
    const int tpc = kWarps / W;
    const int grid = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
    const int n_groups = (pg.nrb + BG - 1) / BG;
    const int cta_groups = cta < n_groups ? (n_groups - cta + grid - 1) / grid : 0;
    auto group_of = [=](int gi) { return cta + (tw + gi * tpc) * grid; };
    const int my_units = (wt < pg.nunits) ? (pg.nunits - wt + W - 1) / W : 0;
    const int my_groups = cta_groups > tw ? (cta_groups - tw + tpc - 1) / tpc : 0;
    const int per_group = BG * my_units;
    const int n_items = my_groups * per_group;

    // The dependent kernel may launch at once: its own PDL wait still waits for this
    // grid to complete, and meanwhile it streams its weights (which depend on nothing).
    pdl_launch_dependents();
    if (lane == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(my_bar0 + 8 * s, 1);
        mbar_init_fence();
    }
    __syncwarp();

    // Issue cursor: the next item to copy, as (group, block, unit) counters of this
    // warp's item order; advanced like an odometer (no divisions per item).
    int ig = 0, ij = 0, iu = 0, n_issued = 0;
    auto issue_next = [&]() {
        const int rb = group_of(ig) * BG + ij;
        const int unit = wt + iu * W;
        const int s = n_issued % kStages;
        const uint32_t bar = my_bar0 + 8 * s;
        if (lane == 0) {
            if (rb < pg.nrb) {
                const unsigned char* src = packed + rb * pg.rb_bytes + static_cast<long long>(unit) * kItemMax;
                const uint32_t bytes =
                    (unit == pg.nunits - 1) ? static_cast<uint32_t>(pg.item_last) : static_cast<uint32_t>(kItemMax);
                mbar_expect_tx(bar, bytes);
                bulk_g2s_hint(smem_u32(my_ring + s * kItemMax), src, bytes, bar, l2_evict_first());
            } else {
                // a padding block of an odd block count: complete the phase without data
                mbar_arrive(bar);
            }
        }
        ++n_issued;
        if (++iu == my_units) {
            iu = 0;
            if (++ij == BG) {
                ij = 0;
                ++ig;
            }
        }
    };
    // weights do not depend on the previous kernel: the first stage before the PDL wait,
    // the others once the input's loads are issued (all of them before the wait when the
    // input arrives through the fused all-reduce, whose wait would delay them)
    const int pre = (AR && p.ar_mode == 2) ? kStages : 1;
    while (n_issued < pre && n_issued < n_items) issue_next();
    PrologueWeights pw;
    if (p.prologue != QmvPrologue::kNone) pw = load_prologue_weights(p);

    pdl_wait();
    if (threadIdx.x < 32) zero_page[threadIdx.x] = 0u;
    stage_input<AR>(p, pw, xp, xsum, tmp, [&]() {
        while (n_issued < kStages && n_issued < n_items) issue_next();
    });
    __syncthreads();

    uint32_t phase_bits = 0;  // one parity bit per stage
    int buf = 0, it = 0;
    float gate0 = 0.f, gate1 = 0.f;  // team = 1 GEGLU: this lane's gate rows g, g + 8
    for (int gi = 0; gi < my_groups; ++gi) {
        const int grp = group_of(gi);
        for (int j = 0; j < BG; ++j) {
            const int rb = grp * BG + j;
            float acc0 = 0.f, acc1 = 0.f;
            for (int ui = 0; ui < my_units; ++ui, ++it) {
                const int unit = wt + ui * W;
                const int s = it % kStages;
                const bool ok = mbar_wait(my_bar0 + 8 * s, (phase_bits >> s) & 1u);
                phase_bits ^= (1u << s);
                // Refill this item's stage with item it + kStages as soon as its bytes are
                // in registers (every lane's reads ordered before lane 0's bulk copy), so
                // two items stay in flight while this one is computed.
                auto refill = [&]() {
                    if (n_issued < n_items) {
                        fence_proxy_async();
                        __syncwarp();
                        issue_next();
                    }
                };
                if (!ok || rb >= pg.nrb) {
                    refill();
                    continue;
                }
                const unsigned char* st = my_ring + s * kItemMax;
                // Full units (8 groups: every lane valid) take a path without the
                // per-lane validity selects; only the last unit can be partial.
                if (unit != pg.nunits - 1 || pg.gc_last == 8)
                    qmv_item<true>(st, xp, zero_page, xsum, pg, unit, g, t, acc0, acc1, refill);
                else
                    qmv_item<false>(st, xp, zero_page, xsum, pg, unit, g, t, acc0, acc1, refill);
            }
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
            if (W == 1) {
                // the warp holds the whole sums: lane (g, 0) has rows g and g + 8
                if (AR && !GEGLU && p.ar_mode == 1) {
                    // even g pairs its rows with rows g + 1 and g + 9 from lane (g + 1, 0)
                    const float n0 = __shfl_down_sync(0xffffffffu, acc0, 4);
                    const float n1 = __shfl_down_sync(0xffffffffu, acc1, 4);
                    if (t == 0 && (g & 1) == 0) {
                        if (rb * 16 + g < pg.N) ar_store_pair(p, rb * 16 + g, f2bf(acc0), f2bf(n0));
                        if (rb * 16 + g + 8 < pg.N) ar_store_pair(p, rb * 16 + g + 8, f2bf(acc1), f2bf(n1));
                    }
                }
                if (t == 0) {
                    if (!GEGLU) {
                        if (rb * 16 + g < pg.N) p.y[rb * 16 + g] = f2bf(acc0);
                        if (rb * 16 + g + 8 < pg.N) p.y[rb * 16 + g + 8] = f2bf(acc1);
                    } else if (j == 0) {
                        gate0 = acc0;
                        gate1 = acc1;
                    } else {
                        const int row = grp * 16 + g;
                        if (row < pg.N / 2) p.y[row] = f2bf(gelu_tanh_bf16ops(rbf(gate0)) * rbf(acc0));
                        if (row + 8 < pg.N / 2) p.y[row + 8] = f2bf(gelu_tanh_bf16ops(rbf(gate1)) * rbf(acc1));
                    }
                }
                continue;
            }
            if (t == 0) {
                red[(buf * kWarps + warp) * 16 + g] = acc0;
                red[(buf * kWarps + warp) * 16 + g + 8] = acc1;
            }
            team_sync(1 + tw, 32 * W);
            if (wt == 0 && lane < 16) {
                float v = 0.f;
                for (int w = 0; w < W; ++w) v += red[(buf * kWarps + tw * W + w) * 16 + lane];
                float* pb = pairbuf + tw * 32;
                if (!GEGLU) {
                    const int row = rb * 16 + lane;
                    if (row < pg.N) p.y[row] = f2bf(v);
                    if (AR && p.ar_mode == 1) {
                        // even lanes pair their row with the next lane's (lanes 0..15 active)
                        const float nv = __shfl_down_sync(0x0000ffffu, v, 1);
                        if ((lane & 1) == 0 && row < pg.N) ar_store_pair(p, row, f2bf(v), f2bf(nv));
                    }
                } else {
                    pb[j * 16 + lane] = v;  // j = 0 gate rows, j = 1 up rows
                    if (j == 1) {
                        const float gv = pb[lane];
                        const int row = grp * 16 + lane;
                        if (row < pg.N / 2) p.y[row] = f2bf(gelu_tanh_bf16ops(rbf(gv)) * rbf(v));
                    }
                }
            }
            buf ^= 1;
        }
    }
}

__global__ void qmv_pack_kernel(const uint32_t* __restrict__ w, const bf16* __restrict__ s,
                                const bf16* __restrict__ b, int K, int N, unsigned char* __restrict__ out) {
    const PackGeo pg = pack_geo(K, N);
    // one thread per (row block, unit, rank): writes its 8 weight chunks and its record
    const long long total = static_cast<long long>(pg.nrb) * pg.nunits * 32;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int L = static_cast<int>(idx % 32);
        const long long ru = idx / 32;
        const int unit = static_cast<int>(ru % pg.nunits);
        const int rb = static_cast<int>(ru / pg.nunits);
        const int gc = (unit == pg.nunits - 1) ? pg.gc_last : 8;
        const int tv = (gc + 1) / 2;
        const int nv = 8 * tv;
        const int g = L / 4, t = L % 4;
        if (t >= tv) continue;
        const int rank = g * tv + t;
        unsigned char* item = out + rb * pg.rb_bytes + static_cast<long long>(unit) * kItemMax;
        const int gA = unit * 8 + 2 * t, gB = gA + 1;
        const int K8 = K / 8, G = pg.G;
        for (int c = 0; c < 8; ++c) {
            const int h = c / 4, q = c % 4;
            const int row = rb * 16 + g + 8 * h;
            const int grp = (q < 2) ? gA : gB;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (row < N && grp < G) v = *reinterpret_cast<const uint4*>(w + static_cast<size_t>(row) * K8 + grp * 8 + 4 * (q & 1));
            *reinterpret_cast<uint4*>(item + (c * nv + rank) * 16) = v;
        }
        uint16_t rec[8];
        for (int h = 0; h < 2; ++h) {
            const int row = rb * 16 + g + 8 * h;
            const bool vr = row < N;
            const uint16_t* sr = reinterpret_cast<const uint16_t*>(s) + static_cast<size_t>(row) * G;
            const uint16_t* br = reinterpret_cast<const uint16_t*>(b) + static_cast<size_t>(row) * G;
            rec[2 * h + 0] = (vr && gA < G) ? sr[gA] : 0;
            rec[2 * h + 1] = (vr && gB < G) ? sr[gB] : 0;
            rec[4 + 2 * h + 0] = (vr && gA < G) ? br[gA] : 0;
            rec[4 + 2 * h + 1] = (vr && gB < G) ? br[gB] : 0;
        }
        *reinterpret_cast<uint4*>(item + (8 * nv + rank) * 16) = *reinterpret_cast<uint4*>(rec);
    }
}

// The inverse of qmv_pack_kernel: the MLX layout (codes [N, K/8] u32, scales and biases
// [N, K/64] bf16) of the rows a packed matrix holds; same thread mapping as the pack.
__global__ void qmv_unpack_kernel(const unsigned char* __restrict__ in, int K, int N, uint32_t* __restrict__ w,
                                  bf16* __restrict__ s, bf16* __restrict__ b) {
    const PackGeo pg = pack_geo(K, N);
    const long long total = static_cast<long long>(pg.nrb) * pg.nunits * 32;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int L = static_cast<int>(idx % 32);
        const long long ru = idx / 32;
        const int unit = static_cast<int>(ru % pg.nunits);
        const int rb = static_cast<int>(ru / pg.nunits);
        const int gc = (unit == pg.nunits - 1) ? pg.gc_last : 8;
        const int tv = (gc + 1) / 2;
        const int nv = 8 * tv;
        const int g = L / 4, t = L % 4;
        if (t >= tv) continue;
        const int rank = g * tv + t;
        const unsigned char* item = in + rb * pg.rb_bytes + static_cast<long long>(unit) * kItemMax;
        const int gA = unit * 8 + 2 * t, gB = gA + 1;
        const int K8 = K / 8, G = pg.G;
        for (int c = 0; c < 8; ++c) {
            const int h = c / 4, q = c % 4;
            const int row = rb * 16 + g + 8 * h;
            const int grp = (q < 2) ? gA : gB;
            if (row < N && grp < G)
                *reinterpret_cast<uint4*>(w + static_cast<size_t>(row) * K8 + grp * 8 + 4 * (q & 1)) =
                    *reinterpret_cast<const uint4*>(item + (c * nv + rank) * 16);
        }
        const uint4 rv = *reinterpret_cast<const uint4*>(item + (8 * nv + rank) * 16);
        const uint16_t* rec = reinterpret_cast<const uint16_t*>(&rv);
        for (int h = 0; h < 2; ++h) {
            const int row = rb * 16 + g + 8 * h;
            if (row >= N) continue;
            uint16_t* sr = reinterpret_cast<uint16_t*>(s) + static_cast<size_t>(row) * G;
            uint16_t* br = reinterpret_cast<uint16_t*>(b) + static_cast<size_t>(row) * G;
            if (gA < G) {
                sr[gA] = rec[2 * h + 0];
                br[gA] = rec[4 + 2 * h + 0];
            }
            if (gB < G) {
                sr[gB] = rec[2 * h + 1];
                br[gB] = rec[4 + 2 * h + 1];
            }
        }
    }
}

// Embedding rows gathered from a packed table (the tied lm_head): row id's group gi lives in
// 16-row block id / 16, unit gi / 8, lane (g = id % 8, t = (gi % 8) / 2) as chunks
// 4 h + 2 (gi % 2) and + 1 (h = (id % 16) / 8) and record entries 2 h + gi % 2 (scale),
// 4 + 2 h + gi % 2 (bias). Dequantised and scaled exactly as embed_kernel does.
__global__ void embed_packed_kernel(const uint32_t* __restrict__ ids, const unsigned char* __restrict__ packed, int H,
                                    int N, bf16 scale, bf16* __restrict__ out) {
    const int l = blockIdx.y;
    const uint32_t id = ids[l];
    const PackGeo pg = pack_geo(H, N);
    const float sc = bf2f(scale);
    const int rb = static_cast<int>(id / 16), rr = static_cast<int>(id % 16), g = rr % 8, h = rr / 8;
    for (int gi = blockIdx.x * blockDim.x + threadIdx.x; gi < pg.G; gi += gridDim.x * blockDim.x) {
        const int unit = gi / 8, t = (gi % 8) / 2, which = gi % 2;
        const int gc = (unit == pg.nunits - 1) ? pg.gc_last : 8;
        const int tv = (gc + 1) / 2, nv = 8 * tv, rank = g * tv + t;
        const unsigned char* item = packed + rb * pg.rb_bytes + static_cast<long long>(unit) * kItemMax;
        const uint4 rv = *reinterpret_cast<const uint4*>(item + (8 * nv + rank) * 16);
        const uint16_t* rec = reinterpret_cast<const uint16_t*>(&rv);
        const float sv = __uint_as_float(static_cast<uint32_t>(rec[2 * h + which]) << 16);
        const float bv = __uint_as_float(static_cast<uint32_t>(rec[4 + 2 * h + which]) << 16);
        for (int half = 0; half < 2; ++half) {
            const int c = 4 * h + 2 * which + half;
            const uint4 wv = *reinterpret_cast<const uint4*>(item + (c * nv + rank) * 16);
            const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
            for (int k = 0; k < 4; ++k) {
                bf16 o[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float deq = rbf(fmaf(sv, static_cast<float>((words[k] >> (4 * i)) & 0xF), bv));
                    o[i] = f2bf(deq * sc);
                }
                *reinterpret_cast<uint4*>(out + static_cast<size_t>(l) * H + gi * 64 + (4 * half + k) * 8) =
                    *reinterpret_cast<uint4*>(o);
            }
        }
    }
}

size_t packed_smem_bytes(int K, bool prologue) {
    const int G = K / 64;
    size_t b = static_cast<size_t>(kWarps) * kStages * kItemMax + kWarps * kStages * 8 +
               static_cast<size_t>(K / 2) * 4 + 32 * 4 + static_cast<size_t>((G + 3) & ~3) * 4 +
               (2 * kWarps * 16 + kWarps * 32 + 32) * 4;  // red, pair, tmp
    (void)prologue;  // the norm prologues work in registers
    return b;
}

}  // namespace

size_t qmv_packed_bytes(int K, int N) {
    const PackGeo pg = pack_geo(K, N);
    return static_cast<size_t>(pg.rb_bytes) * pg.nrb;
}

void launch_qmv_pack(const uint32_t* w, const bf16* s, const bf16* b, int K, int N, void* packed,
                     cudaStream_t stream) {
    if (K <= 0 || K % 64 != 0 || N <= 0) throw ArgError("qmv_pack: K must be a positive multiple of 64");
    const PackGeo pg = pack_geo(K, N);
    const long long total = static_cast<long long>(pg.nrb) * pg.nunits * 32;
    const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 65535));
    qmv_pack_kernel<<<grid, 256, 0, stream>>>(w, s, b, K, N, static_cast<unsigned char*>(packed));
    HYB_LAUNCH_CHECK("qmv_pack_kernel");
}

void launch_qmv_unpack(const void* packed, int K, int N, uint32_t* w, bf16* s, bf16* b, cudaStream_t stream) {
    if (K <= 0 || K % 64 != 0 || N <= 0) throw ArgError("qmv_unpack: K must be a positive multiple of 64");
    const PackGeo pg = pack_geo(K, N);
    const long long total = static_cast<long long>(pg.nrb) * pg.nunits * 32;
    const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 65535));
    qmv_unpack_kernel<<<grid, 256, 0, stream>>>(static_cast<const unsigned char*>(packed), K, N, w, s, b);
    HYB_LAUNCH_CHECK("qmv_unpack_kernel");
}

void launch_embed_packed(const uint32_t* ids, int L, const void* packed, int H, int N, bf16 scale, bf16* out,
                         cudaStream_t stream) {
    if (L <= 0) return;
    if (H % 64 != 0) throw ArgError("embed: hidden size must be a multiple of 64");
    dim3 grid((H / 64 + 63) / 64, L);
    embed_packed_kernel<<<grid, 64, 0, stream>>>(ids, static_cast<const unsigned char*>(packed), H, N, scale, out);
    HYB_LAUNCH_CHECK("embed_packed_kernel");
}

namespace {

void check_packed_stage(const QmvParams& p) {
    if (p.K <= 0 || p.K % 64 != 0 || p.N <= 0) throw ArgError("qmv: K must be a positive multiple of 64");
    if (!p.packed) throw ArgError("qmv_packed: packed weights are required");
    if ((reinterpret_cast<uintptr_t>(p.packed) & 15u) != 0) throw ArgError("qmv_packed: packed weights must be 16-byte aligned");
    const bool pro = p.prologue != QmvPrologue::kNone;
    if (pro && p.K > kMaxPrologueK) throw ArgError("qmv_packed: norm prologues support K <= 8192");
    if (reinterpret_cast<uintptr_t>(p.x) & 15u) throw ArgError("qmv_packed: x must be 16-byte aligned");
    if (packed_smem_bytes(p.K, pro) > 227 * 1024) throw ArgError("qmv_packed: K too large for the shared-memory plan");
    if (p.epilogue == QmvEpilogue::kGeglu && p.N % 32 != 0)
        throw ArgError("qmv geglu: interleaved rows must be a multiple of 32");
}

// Team size: the one with the fewest items on the busiest warp, the smallest on ties
// (independent warps where N is large, the whole CTA on one row block where it is
// small). Returns the team; *grid_needed = CTAs that have work.
int choose_team(const QmvParams& p, int max_ctas, int* grid_needed) {
    const PackGeo pg = pack_geo(p.K, p.N);
    const bool geglu = p.epilogue == QmvEpilogue::kGeglu;
    const int groups = geglu ? (pg.nrb + 1) / 2 : pg.nrb;
    // one CTA per SM at most, each with ceil(groups / grid) groups at most (round-robin)
    const int grid = std::max(1, std::min(groups, max_ctas));
    const int per_cta = (groups + grid - 1) / grid;
    int team = kWarps, best = 1 << 30;
    for (int w = kWarps; w >= 1; w /= 2) {
        const int tpc_w = kWarps / w;
        const int load = (per_cta + tpc_w - 1) / tpc_w * (geglu ? 2 : 1) * ((pg.nunits + w - 1) / w);
        if (load <= best) {
            best = load;
            team = w;
        }
    }
    *grid_needed = grid;
    return team;
}

}  // namespace


void launch_qmv_packed(const QmvParams& p, cudaStream_t stream, bool pdl) {
    check_packed_stage(p);
    if (p.ar_mode != 0) {
        const bool ok_mode = (p.ar_mode == 1 && p.epilogue == QmvEpilogue::kStore &&
                              static_cast<size_t>(p.N) <= p.ar.max_count) ||
                             (p.ar_mode == 2 && p.prologue == QmvPrologue::kResidNorm &&
                              static_cast<size_t>(p.K) <= p.ar.max_count);
        if (!ok_mode || p.ar.T < 2 || p.ar.T > 8 || p.ar.me < 0 || p.ar.me >= p.ar.T)
            throw ArgError("qmv_packed: unsupported fused all-reduce");
    }
    const size_t smem = packed_smem_bytes(p.K, p.prologue != QmvPrologue::kNone);
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    static int attr_dev = -1;
    if (attr_dev != dev) {
        HYB_CUDA(cudaFuncSetAttribute(qmv_packed_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        HYB_CUDA(cudaFuncSetAttribute(qmv_packed_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        HYB_CUDA(cudaFuncSetAttribute(qmv_packed_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        HYB_CUDA(cudaFuncSetAttribute(qmv_packed_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        attr_dev = dev;
    }
    int grid = 1;
    const int team = choose_team(p, kCtasPerSm * num_sms(), &grid);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const bool geglu = p.epilogue == QmvEpilogue::kGeglu, ar = p.ar_mode != 0;
    if (geglu && ar) HYB_CUDA(cudaLaunchKernelEx(&cfg, qmv_packed_kernel<true, true>, p, team));
    else if (geglu) HYB_CUDA(cudaLaunchKernelEx(&cfg, qmv_packed_kernel<true, false>, p, team));
    else if (ar) HYB_CUDA(cudaLaunchKernelEx(&cfg, qmv_packed_kernel<false, true>, p, team));
    else HYB_CUDA(cudaLaunchKernelEx(&cfg, qmv_packed_kernel<false, false>, p, team));
}

int64_t read_qmv_wait_timeouts() {
    int a = 0;
    HYB_CUDA(cudaMemcpyFromSymbol(&a, g_qmv_wait_timeouts, sizeof(int)));
    return a;
}

}  // namespace hyb
