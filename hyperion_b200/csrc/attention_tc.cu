// Prefill (causal, optionally sliding-window) attention on the 5th-generation tensor
// cores: S = Q K^T and O = P V with tcgen05.mma (bf16 operands in shared memory, fp32
// accumulators in TMEM).
//
// Replaces, for prefill chunks, the reference's mx::fast::scaled_dot_product_attention
// call (native/hyperion_mlx/src/forward.cc:498-504) with its bool causal/window mask
// (forward.cc:345-374), evaluated with the MLX CPU-stream rounding: scores rounded to
// bf16 (after the scale and the optional soft-cap), probabilities normalised with the
// row's global max and sum and rounded to bf16 before P V. Exact reproduction needs the
// statistics first, so the key blocks are visited twice: pass 1 only QK^T and the
// running (max, sum); pass 2 QK^T again, p = bf16(exp(s - M) / L) and O += P V.
//
// One CTA: 128 query rows of one head. Warps:
//   0..15 softmax: warp w reads TMEM lanes 32 (w % 4) .. (its 32 query rows) and the
//         16 key columns of quarter w / 4 of each S block with tcgen05.ld; each quarter
//         keeps its (max, sum), merged per row after pass 1; in pass 2 it writes its 16
//         bf16 probabilities of the row into the 128-byte-swizzled K-major P operand;
//         at the end it reads a quarter of its O row and stores bf16;
//   16    TMA producer: the Q tile once, then K tiles (pass 1) and K, V tile pairs
//         (pass 2) of 64 keys into a 4-slot ring;
//   17    allocates TMEM (S double buffer 2 x 64 columns + O hd columns) and issues the
//         MMAs from one thread: S(c + 1) before P V(c), so the softmax of the next block
//         overlaps the product of this one.
// Operands: Q and K tiles are K-major (head_dim contiguous); V tiles are used in place
// as an MN-major B operand (rows = keys, 64 head_dim values per 128-byte row). Every
// mbarrier wait is bounded; TMEM is freed before the CTA exits.
#include "kernels.h"
#include "tcgen05.cuh"
#include "tma.cuh"

#include <algorithm>
#include <cfloat>

namespace hyb {

__device__ int g_attn_tc_wait_timeouts = 0;

namespace {

constexpr int kQRows = 128;
constexpr int kKeys = 64;     // keys per block
constexpr int kSlots = 4;
constexpr int kSoftWarps = 16;                 // 4 TMEM lane groups x 4 key quarters
constexpr int kSoftThreads = kSoftWarps * 32;
constexpr int kThreads = kSoftThreads + 64;    // + TMA warp + MMA warp
constexpr int kTmaWarp = kSoftWarps, kMmaWarp = kSoftWarps + 1;
constexpr int kQCols = kKeys / 4;              // key columns per softmax thread
template <int HD>
struct TcPlan {
    // TMEM: S double buffer (2 x 64 columns) + O (HD columns), rounded to a power of two
    static constexpr uint32_t kTmemCols = HD > 128 ? 512 : 256;
    static constexpr int kQBytes = kQRows * HD * 2;      // HD/64 sub-tiles of [128 rows][128 B]
    static constexpr int kTileBytes = kKeys * HD * 2;    // HD/64 sub-tiles of [64 keys][128 B]
    static constexpr int kPBytes = kQRows * kKeys * 2;   // [128 rows][64 keys] bf16, one sub-tile
    static constexpr int kOffQ = 0;
    static constexpr int kOffSlots = kOffQ + kQBytes;
    static constexpr int kOffP = kOffSlots + kSlots * kTileBytes;
    static constexpr int kOffBars = kOffP + 2 * kPBytes;
    static constexpr int kSmem = kOffBars + 256 + 1024;  // + alignment slack
};

__device__ __forceinline__ bool wait_b(uint32_t bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicAdd(&g_attn_tc_wait_timeouts, 1);
    return false;
}

// Instruction descriptor: bf16 A and B, f32 D; B MN-major when b_mn.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn ? (1u << 16) : 0u) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// MN-major 128-byte-swizzle descriptor: rows are K (keys), 64 N values per 128-byte row;
// 64-wide N groups `lbo` bytes apart, 8-row K groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t smem_addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

__device__ __forceinline__ float score_of(float dot, float scale, float cap, int rounding) {
    float s = dot * scale;
    if (rounding == 0) s = rbf(s);
    if (cap > 0.f) {
        s = cap * tanhf(s / cap);
        if (rounding == 0) s = rbf(s);
    }
    return s;
}

// Thread l of the warp reads TMEM lane (lane field of taddr) + l, 16 consecutive columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// 2^x, flushing denormal results to zero (one MUFU operation): masked scores of -FLT_MAX
// come out as exactly 0.
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void team_sync_n(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

struct TcArgs {
    int Lq, Lk, n_heads, n_kv;
    int q_pos0, k_pos0, window;
    float scale, softcap;
    int rounding;
    bf16* out;
};

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
    using P = TcPlan<HD>;
    constexpr int SUB = HD / 64;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* sm = smem_dyn + ((1024 - (smem_u32(smem_dyn) & 1023)) & 1023);
    const uint32_t sbase = smem_u32(sm);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // causal tiles grow with the query index: every head's longest tiles run first
    // (grid x = heads varies fastest, y = query tiles from the last), a shorter tail wave
    const int q0 = (gridDim.y - 1 - blockIdx.y) * kQRows, h = blockIdx.x;
    const int hk = h / (a.n_heads / a.n_kv);
    const int qrows = min(kQRows, a.Lq - q0);

    // visible key range of the whole tile, in 64-key blocks
    const int qp_lo = a.q_pos0 + q0, qp_hi = a.q_pos0 + q0 + qrows - 1;
    int j_lo = 0;
    if (a.window > 0) j_lo = max(0, qp_lo - a.window + 1 - a.k_pos0);
    const int j_hi = min(a.Lk, qp_hi - a.k_pos0 + 1);  // exclusive
    const int jb0 = (j_lo / kKeys) * kKeys;
    const int nb = j_hi > jb0 ? (j_hi - jb0 + kKeys - 1) / kKeys : 0;

    const uint32_t q_full = sbase + P::kOffBars;
    const uint32_t slot_full = q_full + 8;                // [kSlots]
    const uint32_t slot_empty = slot_full + 8 * kSlots;   // [kSlots]
    const uint32_t s_full = slot_empty + 8 * kSlots;      // [2]
    const uint32_t s_empty = s_full + 16;                 // [2]
    const uint32_t p_full = s_empty + 16;                 // [2]
    const uint32_t p_empty = p_full + 16;                 // [2]
    const uint32_t o_full = p_empty + 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + P::kOffBars + 8 * (2 + 2 * kSlots + 8));

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(slot_full + 8 * s, 1);
            mbar_init(slot_empty + 8 * s, 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(s_full + 8 * s, 1);
            mbar_init(s_empty + 8 * s, kSoftWarps);
            mbar_init(p_full + 8 * s, kSoftWarps);
            mbar_init(p_empty + 8 * s, 1);
        }
        mbar_init(o_full, 1);
        mbar_init_fence();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), P::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_s = tmem;            // S buffers: columns [0, 128)
    const uint32_t tmem_o = tmem + 128;      // O: columns [128, 128 + HD)
    bool ok = true;
    const int n_items = 3 * nb;              // pass 1: nb K tiles; pass 2: nb (K, V) pairs

    if (warp == kTmaWarp) {
        if (lane == 0 && nb > 0) {
            mbar_expect_tx(q_full, P::kQBytes);
#pragma unroll
            for (int d = 0; d < SUB; ++d)
                tma_load_3d(sbase + P::kOffQ + d * (kQRows * 128), &tm_q, 64 * d, h, q0, q_full);
            for (int i = 0; i < n_items; ++i) {
                const int slot = i % kSlots;
                if (i >= kSlots) ok &= wait_b(slot_empty + 8 * slot, ((i / kSlots) - 1) & 1);
                bool is_v;
                int blk;
                if (i < nb) {
                    is_v = false;
                    blk = i;
                } else {
                    is_v = ((i - nb) & 1) != 0;
                    blk = (i - nb) >> 1;
                }
                const int key0 = jb0 + blk * kKeys;
                mbar_expect_tx(slot_full + 8 * slot, P::kTileBytes);
#pragma unroll
                for (int d = 0; d < SUB; ++d)
                    tma_load_3d(sbase + P::kOffSlots + slot * P::kTileBytes + d * (kKeys * 128), is_v ? &tm_v : &tm_k,
                                64 * d, hk, key0, slot_full + 8 * slot);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0 && nb > 0) {
            constexpr uint32_t id_s = idesc_bf16(kQRows, kKeys, false);
            constexpr uint32_t id_o = idesc_bf16(kQRows, HD, true);
            ok &= wait_b(q_full, 0);
            int b = 0;  // S block counter over both passes
            auto issue_s = [&](int item) {
                const int slot = item % kSlots, sb = b & 1;
                ok &= wait_b(slot_full + 8 * slot, (item / kSlots) & 1);
                if (b >= 2) ok &= wait_b(s_empty + 8 * sb, ((b >> 1) - 1) & 1);
                tc_fence_after();
                const uint32_t kbase = sbase + P::kOffSlots + slot * P::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint64_t ad = sw128_kmajor_desc(sbase + P::kOffQ + (kk >> 2) * (kQRows * 128)) + 2 * (kk & 3);
                    const uint64_t bd = sw128_kmajor_desc(kbase + (kk >> 2) * (kKeys * 128)) + 2 * (kk & 3);
                    tc_mma_f16(tmem_s + 64 * sb, ad, bd, id_s, kk > 0 ? 1u : 0u);
                }
                tc_commit(s_full + 8 * sb);
                tc_commit(slot_empty + 8 * slot);
                ++b;
            };
            auto issue_pv = [&](int c, int item) {
                const int slot = item % kSlots, pb = c & 1;
                ok &= wait_b(p_full + 8 * pb, (c >> 1) & 1);
                ok &= wait_b(slot_full + 8 * slot, (item / kSlots) & 1);
                tc_fence_after();
                const uint32_t vbase = sbase + P::kOffSlots + slot * P::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < kKeys / 16; ++kk) {
                    const uint64_t ad = sw128_kmajor_desc(sbase + P::kOffP + pb * P::kPBytes) + 2 * kk;
                    const uint64_t bd = sw128_mnmajor_desc(vbase + kk * 2048, kKeys * 128);
                    tc_mma_f16(tmem_o, ad, bd, id_o, (c > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(p_empty + 8 * pb);
                tc_commit(slot_empty + 8 * slot);
            };
            for (int c = 0; c < nb; ++c) issue_s(c);  // pass 1
            for (int c = 0; c < nb; ++c) {            // pass 2
                issue_s(nb + 2 * c);
                if (c > 0) issue_pv(c - 1, nb + 2 * (c - 1) + 1);
            }
            issue_pv(nb - 1, nb + 2 * (nb - 1) + 1);
            tc_commit(o_full);
        }
    } else {
        // ---------------- softmax warps: warp w reads TMEM lanes 32 (w % 4) .. (its rows) and
        // key columns [16 (w / 4), 16 (w / 4) + 16) of every block; the four quarters of a
        // row keep their own (max, sum), merged once after pass 1
        const int grp = warp & 3, qq = warp >> 2;
        const int r = 32 * grp + lane;
        const int qp = a.q_pos0 + q0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(32 * grp) << 16;
        const float kLog2e = 1.4426950408889634f;
        // keys [kb, kb + 64) visible to every row of the tile: no per-element mask
        auto block_full = [&](int kb) {
            return kb + kKeys <= a.Lk && a.k_pos0 + kb + kKeys - 1 <= qp_lo &&
                   (a.window == 0 || a.k_pos0 + kb > qp_hi - a.window);
        };
        auto load_s = [&](int b, float (&s)[kQCols]) {
            const int sb = b & 1;
            ok &= wait_b(s_full + 8 * sb, (b >> 1) & 1);
            tc_fence_after();
            uint32_t v[kQCols];
            tmem_ld_32x32b_x16(tmem_s + lane_off + 64 * sb + kQCols * qq, v);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_empty + 8 * sb);
#pragma unroll
            for (int i = 0; i < kQCols; ++i) s[i] = score_of(__uint_as_float(v[i]), a.scale, a.softcap, a.rounding);
        };
        auto mask = [&](int kb, float (&s)[kQCols]) {
#pragma unroll
            for (int i = 0; i < kQCols; ++i) {
                const int j = kb + kQCols * qq + i;
                const int kp = a.k_pos0 + j;
                if (!(j < a.Lk && kp <= qp && (a.window == 0 || kp > qp - a.window))) s[i] = -FLT_MAX;
            }
        };
        float m = -FLT_MAX, l = 0.f;
        int b = 0;
        if (nb > 0) {
            // ---- pass 1: this quarter's running max and sum
            for (int c = 0; c < nb; ++c, ++b) {
                float s[kQCols];
                load_s(b, s);
                const int kb = jb0 + c * kKeys;
                if (!block_full(kb)) mask(kb, s);
                float mx = m;
#pragma unroll
                for (int i = 0; i < kQCols; ++i) mx = fmaxf(mx, s[i]);
                if (mx == -FLT_MAX) continue;
                const float ms = mx * kLog2e;  // finite: some key of this quarter is visible
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < kQCols; ++i) acc += ex2_ftz(fmaf(s[i], kLog2e, -ms));  // masked: 0
                l = (m == -FLT_MAX ? 0.f : l * ex2_ftz(fmaf(m, kLog2e, -ms))) + acc;
                m = mx;
            }
            // ---- merge the four quarters of each row (in quarter order: the same on all)
            float* stat = reinterpret_cast<float*>(sm + P::kOffP);  // P buffer 0, free until pass 2
            stat[(qq * kQRows + r) * 2] = m;
            stat[(qq * kQRows + r) * 2 + 1] = l;
            team_sync_n(1, kSoftThreads);
            float M = -FLT_MAX;
#pragma unroll
            for (int u = 0; u < 4; ++u) M = fmaxf(M, stat[(u * kQRows + r) * 2]);
            float L = 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float mu = stat[(u * kQRows + r) * 2], lu = stat[(u * kQRows + r) * 2 + 1];
                if (lu > 0.f) L += lu * ex2_ftz((mu - M) * kLog2e);
            }
            team_sync_n(1, kSoftThreads);  // every thread has read the statistics
            m = M;
            const float il = L > 0.f ? 1.0f / L : 0.f;
            // rows without a visible key (padding rows past Lq) get p = 0 and are not stored
            const float ms = L > 0.f ? m * kLog2e : 0.f;
            // ---- pass 2: probabilities into the P operand (this quarter's 16 keys = 2 chunks)
            for (int c = 0; c < nb; ++c, ++b) {
                float s[kQCols];
                load_s(b, s);
                const int kb = jb0 + c * kKeys;
                if (!block_full(kb)) mask(kb, s);
                const int pb = c & 1;
                if (c >= 2) ok &= wait_b(p_empty + 8 * pb, ((c >> 1) - 1) & 1);
                unsigned char* prow = sm + P::kOffP + pb * P::kPBytes + r * 128;
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    uint32_t w[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float s0 = s[8 * h2 + 2 * q], s1 = s[8 * h2 + 2 * q + 1];
                        const float p0 = ex2_ftz(fmaf(s0, kLog2e, -ms)) * il;  // masked: 0
                        const float p1 = ex2_ftz(fmaf(s1, kLog2e, -ms)) * il;
                        w[q] = pack_bf2(f2bf(p0), f2bf(p1));
                    }
                    const int ch = 2 * qq + h2;
                    *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                }
                fence_proxy_async();  // generic-proxy writes -> the MMA's async-proxy reads
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full + 8 * pb);
            }
            // ---- epilogue: O row -> bf16
            ok &= wait_b(o_full, 0);
            tc_fence_after();
        }
        const bool row_ok = r < qrows;
        bf16* dst = a.out + (static_cast<size_t>(q0 + r) * a.n_heads + h) * HD;
        // this quarter's head_dim columns of the row
#pragma unroll 1
        for (int col = qq * (HD / 4); col < (qq + 1) * (HD / 4); col += 16) {
            uint32_t v[16];
            if (nb > 0) {
                tmem_ld_32x32b_x16(tmem_o + lane_off + col, v);
                tmem_ld_wait();
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = 0u;
            }
            if (row_ok) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    uint4 o;
                    o.x = pack_bf2(f2bf(__uint_as_float(v[8 * q + 0])), f2bf(__uint_as_float(v[8 * q + 1])));
                    o.y = pack_bf2(f2bf(__uint_as_float(v[8 * q + 2])), f2bf(__uint_as_float(v[8 * q + 3])));
                    o.z = pack_bf2(f2bf(__uint_as_float(v[8 * q + 4])), f2bf(__uint_as_float(v[8 * q + 5])));
                    o.w = pack_bf2(f2bf(__uint_as_float(v[8 * q + 6])), f2bf(__uint_as_float(v[8 * q + 7])));
                    *reinterpret_cast<uint4*>(dst + col + 8 * q) = o;
                }
            }
        }
    }
    if (!ok && lane == 0) {
        // a wait gave up: wait (bounded) for copies and MMAs that may still be in flight
        for (int s = 0; s < kSlots && s < n_items; ++s)
            mbar_wait_bounded(slot_full + 8 * s, ((n_items - 1 - s) / kSlots) & 1);
        mbar_wait_bounded(o_full, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, P::kTmemCols);
    }
}

template <int HD>
void launch_tc_t(const PrefillAttnParams& p, cudaStream_t stream) {
    using P = TcPlan<HD>;
    static int attr_dev = -1;
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        HYB_CUDA(cudaFuncSetAttribute(prefill_attn_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, P::kSmem));
        attr_dev = dev;
    }
    CUtensorMap tq, tk, tv;
    {
        const uint64_t dims[3] = {static_cast<uint64_t>(HD), static_cast<uint64_t>(p.n_heads), static_cast<uint64_t>(p.Lq)};
        const uint64_t strides[2] = {static_cast<uint64_t>(HD) * 2, static_cast<uint64_t>(p.n_heads) * HD * 2};
        const uint32_t box[3] = {64, 1, static_cast<uint32_t>(kQRows)};
        encode_tma(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, p.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    {
        const uint64_t dims[3] = {static_cast<uint64_t>(HD), static_cast<uint64_t>(p.n_kv), static_cast<uint64_t>(p.Lk)};
        const uint64_t strides[2] = {static_cast<uint64_t>(HD) * 2, static_cast<uint64_t>(p.n_kv) * HD * 2};
        const uint32_t box[3] = {64, 1, static_cast<uint32_t>(kKeys)};
        encode_tma(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, p.k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        encode_tma(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, p.v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    TcArgs a{p.Lq, p.Lk, p.n_heads, p.n_kv, p.q_pos0, p.k_pos0, p.window, p.scale, p.softcap, p.rounding, p.out};
    dim3 grid(p.n_heads, (p.Lq + kQRows - 1) / kQRows);
    prefill_attn_tc_kernel<HD><<<grid, kThreads, P::kSmem, stream>>>(tq, tk, tv, a);
    HYB_LAUNCH_CHECK("prefill_attn_tc_kernel");
}

}  // namespace

bool prefill_attn_tc_supported(const PrefillAttnParams& p) {
    if (p.hd != 64 && p.hd != 128 && p.hd != 256) return false;
    if (p.Lq <= 0 || p.Lk <= 0 || p.n_kv <= 0 || p.n_heads % p.n_kv != 0) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k) |
                         reinterpret_cast<uintptr_t>(p.v) | reinterpret_cast<uintptr_t>(p.out);
    return (al & 15) == 0;
}

void launch_prefill_attn_tc(const PrefillAttnParams& p, cudaStream_t stream) {
    if (!prefill_attn_tc_supported(p)) throw ArgError("prefill attention (tcgen05): unsupported shape");
    switch (p.hd) {
        case 64: launch_tc_t<64>(p, stream); break;
        case 128: launch_tc_t<128>(p, stream); break;
        default: launch_tc_t<256>(p, stream); break;
    }
}

int64_t read_attn_tc_wait_timeouts() {
    int a = 0;
    HYB_CUDA(cudaMemcpyFromSymbol(&a, g_attn_tc_wait_timeouts, sizeof(int)));
    return a;
}

}  // namespace hyb
