// Batched decode qmv: y[b] = x[b] · Wᵀ for B <= 64 sequences over the packed resident
// weight layout (qmv_pack.cuh), streamed once for the whole batch.
//
// Replaces, for a decode step of B independent sequences, B calls of
// mx::quantized_matmul(transpose=true, group 64, 4 bits, affine) (weights.h:26-37).
//
// The batch-1 kernel folds the per-group scale and bias after the tensor-core product
// (its MMA columns are groups). Here the MMA columns are the sequences, so the codes are
// dequantised in registers first: w = fp16(s·q + b), exact whenever b = −8s (s·(q − 8)
// has at most 11 significant bits), and the activations enter as fp16 (exact for bf16
// values in fp16's normal range). mma.sync m16n8k16 (fp16 in, fp32 accumulate): A = 16
// weight rows × 16 codes, B = 16 codes × 8 sequences. Lane (g, t) of the packed layout
// holds codes of groups 2t, 2t + 1, so an MMA's k dimension spans four groups; the
// weights carry their scales, so that is fine, and lane (n, t) loads the activations of
// sequence n at exactly the code positions lane (·, t) supplies.
//
// x arrives pre-converted (launch_qmv_batched_x16) into fp16 pairs (x[b][8j + p],
// x[b][8j + p + 4]), the nibble pairing of the packed words, tiled so that every warp-wide
// activation load is one contiguous 512-byte run: the 16-byte chunk (pairs p = 0..3 of
// 8-code chunk j = 8G + w, group G = 8u + 2t + sel of unit u, sequence b = 8o + g) sits at
// chunk index ((((u·2 + sel)·8 + w)·NB8 + o)·8 + g)·4 + t, exactly where lane (g, t) of
// MMA column group o reads it; sequences >= B and groups past K are zero. Work split, rings and teams as in the batch-1 kernel; a team sums its warps'
// partials in shared memory in a fixed order.
#include "kernels.h"
#include "qmv_pack.cuh"
#include "tma.cuh"

#include <algorithm>
#include <cuda_fp16.h>

namespace hyb {

__device__ int g_qmvb_wait_timeouts = 0;  // set if an mbarrier wait gave up (never expected)

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 2;

__device__ __forceinline__ bool mbar_wait_b(uint32_t bar, uint32_t phase) {
    if (mbar_wait_bounded(bar, phase)) return true;
    atomicAdd(&g_qmvb_wait_timeouts, 1);
    return false;
}

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// bf16 bits -> fp16 bits, and whether the value is exact in fp16 (normal range or zero).
__device__ __forceinline__ uint16_t bf16_to_h(uint16_t bits, bool& exact) {
    const float f = __uint_as_float(static_cast<uint32_t>(bits) << 16);
    const __half h = __float2half_rn(f);
    exact = exact && (__half2float(h) == f);
    return __half_as_ushort(h);
}

// Dequantised fp16 pair (w[p], w[p + 4]) of a packed word: codes as fp16 1024 + q by the
// exponent trick, minus 1024, times s plus b (one rounding).
__device__ __forceinline__ uint32_t deq_pair(uint32_t word, int p, uint32_t s2, uint32_t b2) {
    const uint32_t q = lop3_and_or(word >> (4 * p), 0x000F000Fu, 0x64006400u);
    return h2_fma(h2_sub(q, 0x64006400u), s2, b2);
}

// Slow path for a (row, group) whose scale or bias is not exact in fp16: the weight in
// fp32, then rounded once to fp16.
__device__ __forceinline__ uint32_t deq_pair_f32(uint32_t word, int p, float s, float b) {
    const float w0 = fmaf(static_cast<float>((word >> (4 * p)) & 15u), s, b);
    const float w1 = fmaf(static_cast<float>((word >> (4 * p + 16)) & 15u), s, b);
    return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(w0))) |
           (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(w1))) << 16);
}

template <bool GEGLU, int NB8>
__global__ void __launch_bounds__(kThreads) qmv_batched_kernel(const QmvBatchParams p, int team) {
    constexpr int BG = GEGLU ? 2 : 1;
    constexpr int BP = NB8 * 8;  // padded batch
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const PackGeo pg = pack_geo(p.K, p.N);
    const unsigned char* packed = static_cast<const unsigned char*>(p.packed);

    // shared memory: [rings kWarps x kStages x 4608][mbar kWarps x kStages][red kWarps x 16 x BP]
    //                [gate (kWarps / team) x 16 x BP]
    unsigned char* ring = smem_raw;
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kWarps * kStages * kItemMax);
    float* red = reinterpret_cast<float*>(bars + kWarps * kStages);
    float* gate = red + kWarps * 16 * BP;
    unsigned char* my_ring = ring + warp * kStages * kItemMax;
    const uint32_t my_bar0 = smem_u32(bars + warp * kStages);

    const int W = team;
    const int tw = warp / W, wt = warp % W;
    // row-block groups are dealt round-robin over the CTAs first, then over the CTA's teams:
    // group_of(i) = cta + (tw + i * tpc) * grid, so every SM holds the same count within one
    const int tpc = kWarps / W, grid = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
    auto group_of = [=](int i) { return cta + (tw + i * tpc) * grid; };
    const int n_groups = (pg.nrb + BG - 1) / BG;
    const int my_units = (wt < pg.nunits) ? (pg.nunits - wt + W - 1) / W : 0;
    const int first = group_of(0);
    const int my_groups = (first < n_groups) ? (n_groups - 1 - first) / (tpc * grid) + 1 : 0;
    const int n_items = my_groups * BG * my_units;

    pdl_launch_dependents();
    if (lane == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(my_bar0 + 8 * s, 1);
        mbar_init_fence();
    }
    __syncwarp();

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
                mbar_arrive(bar);  // a padding block of an odd block count
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
    while (n_issued < kStages && n_issued < n_items) issue_next();
    pdl_wait();

    const uint4* x16q = reinterpret_cast<const uint4*>(p.x16);
    uint32_t phase_bits = 0;
    int it = 0;
    for (int gi = 0; gi < my_groups; ++gi) {
        const int grp = group_of(gi);
        for (int j = 0; j < BG; ++j) {
            const int rb = grp * BG + j;
            float acc[NB8][4];
#pragma unroll
            for (int o = 0; o < NB8; ++o) acc[o][0] = acc[o][1] = acc[o][2] = acc[o][3] = 0.f;
            for (int ui = 0; ui < my_units; ++ui, ++it) {
                const int unit = wt + ui * W;
                const int s = it % kStages;
                const bool ok = mbar_wait_b(my_bar0 + 8 * s, (phase_bits >> s) & 1u);
                phase_bits ^= (1u << s);
                // refill this item's stage with item it + kStages once its bytes are in
                // registers (every lane's reads ordered before lane 0's bulk copy)
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
                const bool full = unit != pg.nunits - 1 || pg.gc_last == 8;
                const int tv = full ? 4 : (pg.gc_last + 1) / 2;
                const int nv = 8 * tv;
                const bool valid = t < tv;
                const int rank = g * tv + t;
                uint4 wv[8];
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    wv[c] = valid ? *reinterpret_cast<const uint4*>(st + (c * nv + rank) * 16) : make_uint4(0, 0, 0, 0);
                const uint4 sb = valid ? *reinterpret_cast<const uint4*>(st + (8 * nv + rank) * 16) : make_uint4(0, 0, 0, 0);
                refill();
#pragma unroll
                for (int sel = 0; sel < 2; ++sel) {  // group 2t (sel 0) or 2t + 1 of the unit
                    const int G = unit * 8 + 2 * t + sel;
                    const bool gvalid = valid && G < pg.G;
                    // record: s = {sA(g), sB(g), sA(g+8), sB(g+8)}, b = {bA(g), bB(g), bA(g+8), bB(g+8)}
                    const uint16_t s0 = static_cast<uint16_t>(sel ? (sb.x >> 16) : (sb.x & 0xFFFFu));
                    const uint16_t s1 = static_cast<uint16_t>(sel ? (sb.y >> 16) : (sb.y & 0xFFFFu));
                    const uint16_t b0 = static_cast<uint16_t>(sel ? (sb.z >> 16) : (sb.z & 0xFFFFu));
                    const uint16_t b1 = static_cast<uint16_t>(sel ? (sb.w >> 16) : (sb.w & 0xFFFFu));
                    bool exact = true;
                    const uint32_t hs0 = bf16_to_h(s0, exact), hs1 = bf16_to_h(s1, exact);
                    const uint32_t hb0 = bf16_to_h(b0, exact), hb1 = bf16_to_h(b1, exact);
                    const uint32_t s2r0 = hs0 | (hs0 << 16), s2r1 = hs1 | (hs1 << 16);
                    const uint32_t b2r0 = hb0 | (hb0 << 16), b2r1 = hb1 | (hb1 << 16);
                    const float fs0 = __uint_as_float(static_cast<uint32_t>(s0) << 16);
                    const float fs1 = __uint_as_float(static_cast<uint32_t>(s1) << 16);
                    const float fb0 = __uint_as_float(static_cast<uint32_t>(b0) << 16);
                    const float fb1 = __uint_as_float(static_cast<uint32_t>(b1) << 16);
                    const bool slow = !__all_sync(0xffffffffu, exact || !gvalid);
                    const uint4* xg = x16q + static_cast<size_t>((unit * 2 + sel) * 8) * NB8 * 32 + lane;
#pragma unroll
                    for (int w = 0; w < 8; ++w) {
                        const uint4 c0 = wv[2 * sel + (w >> 2)], c1 = wv[4 + 2 * sel + (w >> 2)];
                        const int cc = w & 3;
                        const uint32_t wr0 = cc == 0 ? c0.x : cc == 1 ? c0.y : cc == 2 ? c0.z : c0.w;  // row g
                        const uint32_t wr1 = cc == 0 ? c1.x : cc == 1 ? c1.y : cc == 2 ? c1.z : c1.w;  // row g + 8
                        uint32_t a[4][2];  // [pair p][row]
                        if (!slow) {
#pragma unroll
                            for (int pp = 0; pp < 4; ++pp) {
                                a[pp][0] = gvalid ? deq_pair(wr0, pp, s2r0, b2r0) : 0u;
                                a[pp][1] = gvalid ? deq_pair(wr1, pp, s2r1, b2r1) : 0u;
                            }
                        } else {
#pragma unroll
                            for (int pp = 0; pp < 4; ++pp) {
                                a[pp][0] = gvalid ? deq_pair_f32(wr0, pp, fs0, fb0) : 0u;
                                a[pp][1] = gvalid ? deq_pair_f32(wr1, pp, fs1, fb1) : 0u;
                            }
                        }
#pragma unroll
                        for (int o = 0; o < NB8; ++o) {
                            uint4 xv = make_uint4(0, 0, 0, 0);
                            if (gvalid) xv = xg[(w * NB8 + o) * 32];
                            // k-steps: pairs (0, 1) then (2, 3) of word w
                            mma_f16_16816(acc[o], a[0][0], a[0][1], a[1][0], a[1][1], xv.x, xv.y);
                            mma_f16_16816(acc[o], a[2][0], a[2][1], a[3][0], a[3][1], xv.z, xv.w);
                        }
                    }
                }
            }
            // this warp's partial sums: rows g, g + 8; sequences 8o + 2t, 8o + 2t + 1
            float* mine = red + warp * 16 * BP;
#pragma unroll
            for (int o = 0; o < NB8; ++o) {
                const int b = 8 * o + 2 * t;
                mine[g * BP + b] = acc[o][0];
                mine[g * BP + b + 1] = acc[o][1];
                mine[(g + 8) * BP + b] = acc[o][2];
                mine[(g + 8) * BP + b + 1] = acc[o][3];
            }
            team_sync(1 + tw, 32 * W);
            // the team's warps reduce in warp order (the same bits on every run)
            for (int idx = wt * 32 + lane; idx < 16 * BP; idx += 32 * W) {
                const int r = idx / BP, b = idx % BP;
                float v = 0.f;
                for (int w = 0; w < W; ++w) v += red[(tw * W + w) * 16 * BP + idx];
                if (!GEGLU) {
                    const int row = rb * 16 + r;
                    if (b < p.B && row < pg.N) p.y[static_cast<size_t>(b) * p.ldy + row] = f2bf(v);
                } else if (j == 0) {
                    gate[tw * 16 * BP + idx] = v;
                } else {
                    const int row = grp * 16 + r;
                    if (b < p.B && row < pg.N / 2)
                        p.y[static_cast<size_t>(b) * p.ldy + row] =
                            f2bf(gelu_tanh_bf16ops(rbf(gate[tw * 16 * BP + idx])) * rbf(v));
                }
            }
            team_sync(1 + tw, 32 * W);
        }
    }
}

// x [B][ldx] bf16 -> the tiled fp16-pair chunks read by qmv_batched_kernel (one thread per
// 16-byte chunk, padding chunks zero).
__global__ void x16_kernel(const bf16* __restrict__ x, int B, int ldx, int K, int NB8, uint4* __restrict__ x16) {
    const int n_groups = K / 64;
    const long long total = static_cast<long long>((n_groups + 7) / 8) * 512 * NB8;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(i & 3), g = static_cast<int>((i >> 2) & 7);
        long long r = i >> 5;
        const int o = static_cast<int>(r % NB8);
        r /= NB8;
        const int w = static_cast<int>(r & 7), sel = static_cast<int>((r >> 3) & 1), u = static_cast<int>(r >> 4);
        const int b = 8 * o + g, G = 8 * u + 2 * t + sel;
        uint4 out = make_uint4(0, 0, 0, 0);
        if (b < B && G < n_groups) {
            const uint4 v = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(b) * ldx + 8 * (8 * G + w));
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
            float f[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                f[2 * q] = __uint_as_float(wd[q] << 16);
                f[2 * q + 1] = __uint_as_float(wd[q] & 0xFFFF0000u);
            }
            auto h = [](float a) { return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(a))); };
            out.x = h(f[0]) | (h(f[4]) << 16);
            out.y = h(f[1]) | (h(f[5]) << 16);
            out.z = h(f[2]) | (h(f[6]) << 16);
            out.w = h(f[3]) | (h(f[7]) << 16);
        }
        x16[i] = out;
    }
}

template <bool GEGLU, int NB8>
void launch_t(const QmvBatchParams& p, int team, int grid, size_t smem, cudaStream_t stream, bool pdl) {
    auto kern = qmv_batched_kernel<GEGLU, NB8>;
    static int attr_dev = -1;
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        HYB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        attr_dev = dev;
    }
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
    HYB_CUDA(cudaLaunchKernelEx(&cfg, kern, p, team));
}

}  // namespace

size_t qmv_batch_x16_words(int B, int K) {
    return static_cast<size_t>((K / 64 + 7) / 8) * 256 * qmv_batch_pad(B);
}

int qmv_batch_pad(int B) {
    if (B <= 8) return 8;
    if (B <= 16) return 16;
    if (B <= 32) return 32;
    return 64;
}

void launch_qmv_batched_x16(const bf16* x, int B, int ldx, int K, uint32_t* x16, cudaStream_t stream) {
    if (B < 1 || B > kMaxDecodeBatch || K <= 0 || K % 64 != 0 || ldx < K || (ldx % 8) != 0)
        throw ArgError("qmv batched: bad activation shape");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(x16)) & 15u)
        throw ArgError("qmv batched: activations must be 16-byte aligned");
    const int NB8 = qmv_batch_pad(B) / 8;
    const long long total = static_cast<long long>((K / 64 + 7) / 8) * 512 * NB8;
    const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 4 * num_sms()));
    x16_kernel<<<grid, 256, 0, stream>>>(x, B, ldx, K, NB8, reinterpret_cast<uint4*>(x16));
    HYB_LAUNCH_CHECK("x16_kernel");
}

void launch_qmv_batched(const QmvBatchParams& p, cudaStream_t stream, bool pdl) {
    if (p.K <= 0 || p.K % 64 != 0 || p.N <= 0) throw ArgError("qmv batched: K must be a positive multiple of 64");
    if (p.B < 1 || p.B > kMaxDecodeBatch) throw ArgError("qmv batched: batch must be 1..64");
    if (!p.packed || !p.x16 || !p.y) throw ArgError("qmv batched: null operand");
    if ((reinterpret_cast<uintptr_t>(p.packed) | reinterpret_cast<uintptr_t>(p.x16)) & 15u)
        throw ArgError("qmv batched: packed weights and x16 must be 16-byte aligned");
    if (p.geglu && p.N % 32 != 0) throw ArgError("qmv batched geglu: interleaved rows must be a multiple of 32");
    const int outN = p.geglu ? p.N / 2 : p.N;
    if (p.ldy < outN) throw ArgError("qmv batched: output row stride too small");
    const int BP = qmv_batch_pad(p.B);
    const PackGeo pg = pack_geo(p.K, p.N);
    const int groups = p.geglu ? (pg.nrb + 1) / 2 : pg.nrb;
    const size_t smem = static_cast<size_t>(kWarps) * kStages * kItemMax + kWarps * kStages * 8 +
                        static_cast<size_t>(kWarps) * 16 * BP * 4 * 2;  // red + gate
    // CTAs per SM at this shared-memory size (at most 2)
    const int per_sm = smem <= 110 * 1024 ? 2 : 1;
    const int max_ctas = per_sm * num_sms();
    // team size: fewest items on the busiest warp, the smallest team on ties
    // (groups go round-robin over the CTAs, so the busiest CTA holds ceil(groups / grid))
    const int grid = std::max(1, std::min(groups, max_ctas));
    const int per_cta = (groups + grid - 1) / grid;
    int team = kWarps, best = 1 << 30;
    for (int w = kWarps; w >= 1; w /= 2) {
        const int tpc_w = kWarps / w;
        const int load = (per_cta + tpc_w - 1) / tpc_w * (p.geglu ? 2 : 1) * ((pg.nunits + w - 1) / w);
        if (load <= best) {
            best = load;
            team = w;
        }
    }
    switch (BP) {
        case 8: p.geglu ? launch_t<true, 1>(p, team, grid, smem, stream, pdl) : launch_t<false, 1>(p, team, grid, smem, stream, pdl); break;
        case 16: p.geglu ? launch_t<true, 2>(p, team, grid, smem, stream, pdl) : launch_t<false, 2>(p, team, grid, smem, stream, pdl); break;
        case 32: p.geglu ? launch_t<true, 4>(p, team, grid, smem, stream, pdl) : launch_t<false, 4>(p, team, grid, smem, stream, pdl); break;
        default: p.geglu ? launch_t<true, 8>(p, team, grid, smem, stream, pdl) : launch_t<false, 8>(p, team, grid, smem, stream, pdl); break;
    }
}

int64_t read_qmvb_wait_timeouts() {
    int a = 0;
    HYB_CUDA(cudaMemcpyFromSymbol(&a, g_qmvb_wait_timeouts, sizeof(int)));
    return a;
}

}  // namespace hyb
