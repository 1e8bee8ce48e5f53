// Prefill quantized matmul on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Y[M, N] = X[M, K] · dequant(W)[N, K]^T for MLX affine Q4/g64 weights (u32 [N, K/8],
// bf16 scales/biases [N, K/64]) and bf16 activations; the reference's op is
// mx::quantized_matmul with transpose=true (native/hyperion_mlx/src/weights.h:26-37).
//
// X is first converted once to f16 (K-permuted, see below) by a small kernel, so that
// the GEMM's many N tiles all load it straight into their MMA operand rings. One CTA
// computes MT x 128 tokens (MT = 2 when there are enough tiles) by 256 weight rows; K
// advances one 64-wide group per stage:
//   warp 8       TMA producer: MT f16 X blocks [128 x 64] (128-byte swizzle, the MMA's
//                operand layout as is) and the W codes [256 rows x 8 u32] into an
//                S-stage ring (one barrier per stage);
//   warps 0..7   converters: row t's 64 codes to f16 w = s*q + b (one f16x2 fma when s
//                and b are exact in f16, else an fp32 fma; one rounding either way),
//                written K-major in the 128-byte swizzle layout into a 2-stage operand
//                ring; then the epilogue;
//   warp 9       allocates 256 MT TMEM columns and issues, per stage, 4 MT
//                tcgen05.mma.kind::f16 (M = 128, N = 256, K = 16) accumulating in
//                TMEM; tcgen05.commit releases the stages and finally the accumulators.
// Split-K (grid z): when the output tiles cannot fill the GPU (decode-sized M), slice z
// takes k-blocks [z kper, (z + 1) kper) and writes fp32 partials, which a second kernel
// sums in slice order (deterministic) into bf16.
// Operand precision: f16 weights are exact for s*(q - 8) codes and within 2^-12
// otherwise; bf16 weights would add ~2.3e-3 relative error, above the 2e-3 parity bound.
// bf16 activations convert to f16 exactly inside f16's range (|x| < 65504).
// Every mbarrier wait is bounded; TMEM is always freed before the CTA exits.
#include "kernels.h"
#include "qmv_pack.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

#include <algorithm>

namespace hyb {

__device__ int g_qmm_wait_timeouts = 0;

namespace {

constexpr int kBM = 128;           // tokens per MMA (M) and per TMEM lane block
constexpr int kBN = 256;           // weight rows per tile (MMA N)
constexpr int kBK = 64;            // one quantization group per stage
constexpr int kOps = 2;            // f16 weight-operand stages
constexpr int kConvWarps = 8;
constexpr int kConvThreads = kConvWarps * 32;
constexpr int kThreads = kConvThreads + 64;      // + TMA warp + MMA warp
constexpr int kTmaWarp = kConvWarps, kMmaWarp = kConvWarps + 1;
constexpr int kXBytes = kBM * kBK * 2;           // 16 KB per 128-token f16 X block
constexpr int kWRawBytes = kBN * kBK / 2;        // 8 KB of codes
constexpr int kBBytes = kBN * kBK * 2;           // 32 KB of f16 weights
constexpr uint32_t kIdesc = idesc_f16_f32(kBM, kBN);

// MT 128-token blocks per CTA (MT = 2 fills all 512 TMEM columns); S TMA stages.
template <int MT>
struct Plan {
    static constexpr int S = MT == 1 ? 4 : 3;
    static constexpr int kOffA = 0;                                   // [S][MT][16 KB] f16 X (TMA, swizzled)
    static constexpr int kOffB = kOffA + S * MT * kXBytes;            // [kOps][32 KB] f16 W (swizzled)
    static constexpr int kOffW = kOffB + kOps * kBBytes;              // [S][8 KB] codes (TMA, dense rows)
    static constexpr int kOffBars = kOffW + S * kWRawBytes;
    static constexpr int kSmem = kOffBars + 256 + 1024;               // + alignment slack
};

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicAdd(&g_qmm_wait_timeouts, 1);
    return false;
}

// byte offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<const uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<const __half2*>(&v); }

// K order inside each 8-element chunk of both operands: f16 pair p holds elements
// (p, p + 4), p = 0..3. The MMA sums over K in any consistent order, and this one lets a
// single lop3 take codes p and p + 4 of a packed word (bits [4p, 4p+4) and [4p+16, 4p+20)).
__global__ void x_to_f16_perm_kernel(const uint4* __restrict__ x, uint4* __restrict__ xh, size_t n_chunks) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n_chunks;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint4 v = x[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};  // (x0,x1) (x2,x3) (x4,x5) (x6,x7)
        uint4 o;
        o.x = h2_bits(__floats2half2_rn(__uint_as_float(w[0] << 16), __uint_as_float(w[2] << 16)));
        o.y = h2_bits(__floats2half2_rn(__uint_as_float(w[0] & 0xFFFF0000u), __uint_as_float(w[2] & 0xFFFF0000u)));
        o.z = h2_bits(__floats2half2_rn(__uint_as_float(w[1] << 16), __uint_as_float(w[3] << 16)));
        o.w = h2_bits(__floats2half2_rn(__uint_as_float(w[1] & 0xFFFF0000u), __uint_as_float(w[3] & 0xFFFF0000u)));
        xh[i] = o;
    }
}

// Dequantise 4 packed words (32 codes) of one weight row into 4 swizzled 16-byte chunks.
template <bool F16>
__device__ __forceinline__ void dequant4(const uint32_t (&words)[4], float sv, float bv, __half sh, __half bh,
                                         unsigned char* row_base, int r, int c0) {
    const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        uint32_t h[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            // (1024 + q_p, 1024 + q_{p+4}) as an f16 pair, then the exact codes
            const uint32_t m = lop3_and_or(words[jj] >> (4 * p), 0x000F000Fu, 0x64006400u);
            const __half2 q = __hsub2(bits_h2(m), k1024);
            if (F16) {
                h[p] = h2_bits(__hfma2(q, __half2(sh, sh), __half2(bh, bh)));  // one rounding
            } else {
                const float2 qf = __half22float2(q);
                h[p] = h2_bits(__floats2half2_rn(fmaf(sv, qf.x, bv), fmaf(sv, qf.y, bv)));
            }
        }
        *reinterpret_cast<uint4*>(row_base + sw128(r, c0 + jj)) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1)
    qmm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                  const bf16* __restrict__ scales, const bf16* __restrict__ biases, bf16* __restrict__ y, int M,
                  int K, int N, int kper, float* __restrict__ part, int geglu) {
    using P = Plan<MT>;
    constexpr int S = P::S;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* sm = smem_dyn + ((1024 - (smem_u32(smem_dyn) & 1023)) & 1023);
    const uint32_t sbase = smem_u32(sm);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kBM * MT, n0 = blockIdx.y * kBN;
    const int k_first = static_cast<int>(blockIdx.z) * kper;       // this slice's k-blocks
    const int nk = min(K / kBK - k_first, kper);                  // >= 1 by construction
    const int G = K / 64;

    const uint32_t tma_full = sbase + P::kOffBars;  // [S]: X blocks and W codes landed
    const uint32_t tma_empty = tma_full + 8 * S;    // [S]: converters read the codes and the MMAs read X
    const uint32_t b_full = tma_empty + 8 * S;      // [kOps]: f16 weights written
    const uint32_t b_empty = b_full + 8 * kOps;     // [kOps]: the MMAs that read them completed
    const uint32_t acc_full = b_empty + 8 * kOps;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + P::kOffBars + 8 * (2 * S + 2 * kOps + 1));

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(tma_full + 8 * s, 1);
            mbar_init(tma_empty + 8 * s, kConvWarps + 1);
        }
        for (int s = 0; s < kOps; ++s) {
            mbar_init(b_full + 8 * s, kConvWarps);
            mbar_init(b_empty + 8 * s, 1);
        }
        mbar_init(acc_full, 1);
        mbar_init_fence();
    }
    if (warp == kMmaWarp) {  // the MMA warp owns the accumulators' TMEM
        tmem_alloc(smem_u32(tmem_slot), kBN * MT);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == kTmaWarp) {
        // ---------------- TMA producer
        if (lane == 0) {
            for (int kt = 0; kt < nk; ++kt) {
                const int s = kt % S;
                if (kt >= S) ok &= wait_bar(tma_empty + 8 * s, ((kt / S) - 1) & 1);
                mbar_expect_tx(tma_full + 8 * s, MT * kXBytes + kWRawBytes);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                    tma_load_2d(sbase + P::kOffA + (s * MT + mt) * kXBytes, &tm_x, (k_first + kt) * kBK,
                                m0 + kBM * mt, tma_full + 8 * s);
                tma_load_2d(sbase + P::kOffW + s * kWRawBytes, &tm_w, (k_first + kt) * (kBK / 8), n0,
                            tma_full + 8 * s);
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer
        if (lane == 0) {
            for (int kt = 0; kt < nk; ++kt) {
                const int s = kt % S, sb = kt % kOps;
                ok &= wait_bar(tma_full + 8 * s, (kt / S) & 1);
                ok &= wait_bar(b_full + 8 * sb, (kt / kOps) & 1);
                tc_fence_after();
                const uint64_t bd = sw128_kmajor_desc(sbase + P::kOffB + sb * kBBytes);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint64_t ad = sw128_kmajor_desc(sbase + P::kOffA + (s * MT + mt) * kXBytes);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)  // +32 bytes (2 descriptor units) per K step
                        tc_mma_f16(tmem + kBN * mt, ad + 2 * k, bd + 2 * k, kIdesc, (kt > 0 || k > 0) ? 1u : 0u);
                }
                tc_commit(tma_empty + 8 * s);  // X blocks of this stage consumed
                tc_commit(b_empty + 8 * sb);   // f16 weights of this stage consumed
            }
            tc_commit(acc_full);  // the accumulators are complete
        }
    } else {
        // ---------------- converters (warps 0..7): row t of the weight tile, then the epilogue
        const int t = threadIdx.x;  // 0..255
        const int n = n0 + t;
        const bool row_ok = n < N;
        const bf16* srow = scales + static_cast<size_t>(row_ok ? n : 0) * G + k_first;
        const bf16* brow = biases + static_cast<size_t>(row_ok ? n : 0) * G + k_first;
        // scale/bias ring: slot (kt mod 4) holds stage kt, loaded three stages ahead
        float sr[4] = {0.f, 0.f, 0.f, 0.f}, br[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int u = 0; u < 3; ++u)
            if (row_ok && u < nk) {
                sr[u] = bf2f(srow[u]);
                br[u] = bf2f(brow[u]);
            }
        for (int kb = 0; kb < nk; kb += 4) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int kt = kb + u;
                if (kt >= nk) break;
                const int s = kt % S, sb = u & 1;  // kOps = 2 and kb is a multiple of 4
                if (row_ok && kt + 3 < nk) {
                    sr[(u + 3) & 3] = bf2f(srow[kt + 3]);
                    br[(u + 3) & 3] = bf2f(brow[kt + 3]);
                }
                ok &= wait_bar(tma_full + 8 * s, (kt / S) & 1);
                if (kt >= kOps) ok &= wait_bar(b_empty + 8 * sb, ((kt / kOps) - 1) & 1);
                tc_fence_after();
                const uint4* wr = reinterpret_cast<const uint4*>(sm + P::kOffW + s * kWRawBytes + t * 32);
                const uint4 w01 = wr[0], w23 = wr[1];
                const uint32_t wa[4] = {w01.x, w01.y, w01.z, w01.w}, wb[4] = {w23.x, w23.y, w23.z, w23.w};
                __syncwarp();
                if (lane == 0) mbar_arrive(tma_empty + 8 * s);  // codes are in registers
                unsigned char* bb = sm + P::kOffB + sb * kBBytes;
                const float sv = sr[u], bv = br[u];
                const __half sh = __float2half_rn(sv), bh = __float2half_rn(bv);
                if (__half2float(sh) == sv && __half2float(bh) == bv) {
                    dequant4<true>(wa, sv, bv, sh, bh, bb, t, 0);
                    dequant4<true>(wb, sv, bv, sh, bh, bb, t, 4);
                } else {
                    dequant4<false>(wa, sv, bv, sh, bh, bb, t, 0);
                    dequant4<false>(wb, sv, bv, sh, bh, bb, t, 4);
                }
                fence_proxy_async();  // generic-proxy operand writes -> the MMA's async-proxy reads
                __syncwarp();
                if (lane == 0) mbar_arrive(b_full + 8 * sb);
            }
        }
        // ---------------- epilogue: TMEM lanes 32 (warp % 4) .. are this warp's tokens
        ok &= wait_bar(acc_full, 0);
        tc_fence_after();
        const int quarter = warp & 3, half = warp >> 2;  // 128 columns per warp and block
#pragma unroll 1
        for (int mt = 0; mt < MT; ++mt) {
            const int m = m0 + kBM * mt + 32 * quarter + lane;
#pragma unroll 1
            for (int j = 0; j < 4; ++j) {
                const int col = 128 * half + 32 * j;
                uint32_t rr[32];
                tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * quarter) << 16) +
                                       static_cast<uint32_t>(kBN * mt + col),
                                   rr);
                tmem_ld_wait();
                if (m < M && part) {
                    float* dst = part + (static_cast<size_t>(blockIdx.z) * M + m) * N + n0 + col;
                    if (n0 + col + 32 <= N && (N % 4) == 0) {
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            *reinterpret_cast<uint4*>(dst + 4 * v) =
                                make_uint4(rr[4 * v], rr[4 * v + 1], rr[4 * v + 2], rr[4 * v + 3]);
                    } else {
                        for (int v = 0; v < 32; ++v)
                            if (n0 + col + v < N) dst[v] = __uint_as_float(rr[v]);
                    }
                } else if (m < M && geglu) {
                    // interleaved gate/up: these 32 columns are one 16-row gate tile and its
                    // up tile, i.e. outputs (n0 + col) / 2 .. + 15 of the GeGLU row
                    if (n0 + col + 32 <= N) {
                        bf16* dst = y + static_cast<size_t>(m) * (N / 2) + (n0 + col) / 2;
#pragma unroll
                        for (int v = 0; v < 2; ++v) {
                            float o[8];
#pragma unroll
                            for (int r = 0; r < 8; ++r) {
                                const float gv = rbf(__uint_as_float(rr[8 * v + r]));
                                const float uv = rbf(__uint_as_float(rr[16 + 8 * v + r]));
                                o[r] = gelu_tanh_bf16ops(gv) * uv;
                            }
                            uint4 q;
                            q.x = pack_bf2(f2bf(o[0]), f2bf(o[1]));
                            q.y = pack_bf2(f2bf(o[2]), f2bf(o[3]));
                            q.z = pack_bf2(f2bf(o[4]), f2bf(o[5]));
                            q.w = pack_bf2(f2bf(o[6]), f2bf(o[7]));
                            *reinterpret_cast<uint4*>(dst + 8 * v) = q;
                        }
                    }
                } else if (m < M) {
                    bf16* dst = y + static_cast<size_t>(m) * N + n0 + col;
                    if (n0 + col + 32 <= N && (N % 8) == 0) {
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            uint4 o;
                            o.x = pack_bf2(f2bf(__uint_as_float(rr[8 * v + 0])), f2bf(__uint_as_float(rr[8 * v + 1])));
                            o.y = pack_bf2(f2bf(__uint_as_float(rr[8 * v + 2])), f2bf(__uint_as_float(rr[8 * v + 3])));
                            o.z = pack_bf2(f2bf(__uint_as_float(rr[8 * v + 4])), f2bf(__uint_as_float(rr[8 * v + 5])));
                            o.w = pack_bf2(f2bf(__uint_as_float(rr[8 * v + 6])), f2bf(__uint_as_float(rr[8 * v + 7])));
                            *reinterpret_cast<uint4*>(dst + 8 * v) = o;
                        }
                    } else {
                        for (int v = 0; v < 32; ++v)
                            if (n0 + col + v < N) dst[v] = f2bf(__uint_as_float(rr[v]));
                    }
                }
            }
        }
    }
    if (!ok && lane == 0) {
        // a wait gave up: wait (bounded) for copies and MMAs that may still be in flight
        for (int s = 0; s < S && s < nk; ++s) mbar_wait_bounded(tma_full + 8 * s, ((nk - 1 - s) / S) & 1);
        mbar_wait_bounded(acc_full, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kBN * MT);
    }
}

// y[m][n] = bf16(sum over slices z of part[z][m][n]), in slice order.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, size_t mn, bf16* __restrict__ y) {
    for (size_t i = (blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x) * 4; i < mn;
         i += static_cast<size_t>(gridDim.x) * blockDim.x * 4) {
        if (i + 4 <= mn && (mn & 3) == 0) {  // every slice's row of 4 stays 16-byte aligned
            float4 a = *reinterpret_cast<const float4*>(part + i);
            for (int z = 1; z < splits; ++z) {
                const float4 v = *reinterpret_cast<const float4*>(part + z * mn + i);
                a.x += v.x;
                a.y += v.y;
                a.z += v.z;
                a.w += v.w;
            }
            *reinterpret_cast<uint2*>(y + i) = make_uint2(pack_bf2(f2bf(a.x), f2bf(a.y)), pack_bf2(f2bf(a.z), f2bf(a.w)));
        } else {
            for (size_t j = i; j < mn && j < i + 4; ++j) {
                float a = part[j];
                for (int z = 1; z < splits; ++z) a += part[z * mn + j];
                y[j] = f2bf(a);
            }
        }
    }
}

template <int MT>
void launch_tc(const CUtensorMap& tx, const CUtensorMap& tw, const bf16* s, const bf16* b, bf16* y, int M, int K,
               int N, int splits, int kper, float* part, bool geglu, cudaStream_t stream) {
    static int attr_dev = -1;
    int dev = 0;
    HYB_CUDA(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        HYB_CUDA(cudaFuncSetAttribute(qmm_tc_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, Plan<MT>::kSmem));
        attr_dev = dev;
    }
    const dim3 grid((M + kBM * MT - 1) / (kBM * MT), (N + kBN - 1) / kBN, splits);
    qmm_tc_kernel<MT><<<grid, kThreads, Plan<MT>::kSmem, stream>>>(tx, tw, s, b, y, M, K, N, kper, part,
                                                                  geglu ? 1 : 0);
    HYB_LAUNCH_CHECK("qmm_tc_kernel");
}

}  // namespace

bool qmm_tc_supported(int M, int K, int N) {
    return M >= 2 && K >= 64 && K % 64 == 0 && N >= 1;
}

namespace {

// The tile plan of an M x N x K product: 2 or 1 token blocks per CTA, or split-K (0).
int tc_plan(int M, int K, int N) {
    const long long tiles2 = static_cast<long long>((M + 255) / 256) * ((N + kBN - 1) / kBN);
    const long long tiles1 = static_cast<long long>((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
    const int nk = K / kBK;
    if (tiles2 >= num_sms()) return 2;
    if (tiles1 >= num_sms() || nk < 8) return 1;
    return 0;
}

}  // namespace

bool qmm_tc_geglu_supported(int M, int K, int N) {
    return qmm_tc_supported(M, K, N) && N % 32 == 0 && tc_plan(M, K, N) != 0;
}

void launch_qmm_tc(const bf16* x, const uint32_t* w, const bf16* s, const bf16* b, bf16* y, int M, int K, int N,
                   cudaStream_t stream, bool geglu) {
    if (!qmm_tc_supported(M, K, N)) throw ArgError("qmm: shape not supported by the tensor-core path");
    if (geglu && !qmm_tc_geglu_supported(M, K, N)) throw ArgError("qmm: GeGLU epilogue not supported for this shape");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15)
        throw ArgError("qmm: x and w must be 16-byte aligned");
    // X to f16 (K-permuted) once; every N tile then loads it straight into the MMA operand ring
    const size_t xh_bytes = static_cast<size_t>(M) * K * 2;
    void* xh = nullptr;
    HYB_CUDA(cudaMallocAsync(&xh, xh_bytes, stream));
    const size_t chunks = xh_bytes / 16;
    const int cgrid = static_cast<int>(std::min<size_t>((chunks + 255) / 256, 4 * static_cast<size_t>(num_sms())));
    x_to_f16_perm_kernel<<<cgrid, 256, 0, stream>>>(reinterpret_cast<const uint4*>(x), static_cast<uint4*>(xh), chunks);
    HYB_LAUNCH_CHECK("x_to_f16_perm_kernel");
    CUtensorMap tx, tw;
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
        const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
        const uint32_t box[2] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(kBM)};
        encode_tma(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(K / 8), static_cast<uint64_t>(N)};
        const uint64_t strides[1] = {static_cast<uint64_t>(K) / 2};
        const uint32_t box[2] = {static_cast<uint32_t>(kBK / 8), static_cast<uint32_t>(kBN)};
        encode_tma(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    // two 128-token blocks per CTA once there are enough tiles to fill the GPU
    const long long tiles1 = static_cast<long long>((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
    const int nk = K / kBK;
    const int plan = tc_plan(M, K, N);
    if (plan == 2) {
        launch_tc<2>(tx, tw, s, b, y, M, K, N, 1, nk, nullptr, geglu, stream);
    } else if (plan == 1) {
        launch_tc<1>(tx, tw, s, b, y, M, K, N, 1, nk, nullptr, geglu, stream);
    } else {
        // split K so that about two CTAs per SM work, each slice at least 4 k-blocks
        int splits = static_cast<int>(std::min<long long>(nk / 4, (2LL * num_sms() + tiles1 - 1) / tiles1));
        splits = std::max(splits, 1);
        const int kper = (nk + splits - 1) / splits;
        splits = (nk + kper - 1) / kper;  // no empty slice
        const size_t mn = static_cast<size_t>(M) * N;
        float* part = nullptr;
        HYB_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&part), mn * splits * sizeof(float), stream));
        launch_tc<1>(tx, tw, s, b, y, M, K, N, splits, kper, part, false, stream);
        const int rgrid = static_cast<int>(std::min<size_t>((mn / 4 + 255) / 256 + 1, 8 * static_cast<size_t>(num_sms())));
        splitk_reduce_kernel<<<rgrid, 256, 0, stream>>>(part, splits, mn, y);
        HYB_LAUNCH_CHECK("splitk_reduce_kernel");
        HYB_CUDA(cudaFreeAsync(part, stream));
    }
    HYB_CUDA(cudaFreeAsync(xh, stream));
}

int64_t read_qmm_wait_timeouts() {
    int a = 0;
    HYB_CUDA(cudaMemcpyFromSymbol(&a, g_qmm_wait_timeouts, sizeof(int)));
    return a;
}

}  // namespace hyb
