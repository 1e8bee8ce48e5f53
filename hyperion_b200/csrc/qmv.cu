// Batch-1 affine Q4/g64 quantized matvec (the decode projection kernel).
//
// Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4,
// "affine") with M == 1 as called from QuantizedLinear::apply
// (native/hyperion_mlx/src/weights.h:26-37) for q/k/v/o, gate/up/down and the
// tied lm_head (forward.cc:137-152, 338-343, 395-412, 507).
//
// Math: y[n] = sum_g s[n,g] * sum_{k in g} q[n,k] x[k] + b[n,g] * sum_{k in g} x[k].
// The per-group integer dot products run on the tensor cores (mma.sync m16n8k16,
// bf16 operands, fp32 accumulate) so that dequantisation costs ~1 instruction per
// nibble instead of ~3 on the CUDA cores:
//   * A operand = the codes, turned into bf16 with one lop3 per nibble pair:
//     (w >> 4p) & 0x000F000F | 0x43004300 gives the bf16 pair (128 + q_p, 128 + q_{p+4}).
//     The +128 offset is folded into the bias term: s*(D - 128*xsum) + b*xsum.
//   * B operand = the activation, but column c of the 16x8 tile only carries the
//     x values of group c of the current 512-wide k unit, so D[:, c] ends up holding
//     that group's dot product and no per-group accumulator reset is needed.
//   * Lane (g = lane/4, t = lane%4) loads, for rows g and g+8 of a 16-row tile, the
//     64 contiguous bytes of groups 2t and 2t+1 of the unit (4 x 128-bit loads per
//     row; the warp reads 16 rows x 256 contiguous bytes). Pair p of word i of group
//     2t feeds A k-slots {2t,2t+1}; the same pair of group 2t+1 feeds slots
//     {2t+8,2t+9}; so D[g][2t], D[g][2t+1] come out in exactly the lane that holds
//     those groups' scales.
// Each CTA (8 warps) owns 16*RT rows at a time; its warps split the k units and
// are reduced through shared memory. Weight loads for the next work item are
// issued before the current one is computed (register double buffering), and the
// first item's loads are issued before the programmatic-dependent-launch wait.
#include "kernels.h"

#include <algorithm>

namespace hyb {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

template <int RT>
struct Item {
    uint4 w[RT][2][4];   // [tile][row g / g+8][gA lo, gA hi, gB lo, gB hi]
    uint32_t s[RT][2];   // bf16 pair (s[gA], s[gB]) per row
    uint32_t b[RT][2];
};

struct Geo {
    int K, N, G, nunits, nrb, rows_per_block;
};

template <int RT>
__device__ __forceinline__ void load_item(Item<RT>& it, const QmvParams& p, const Geo& geo, int rb,
                                          int unit, int g, int t) {
    const int gA = unit * 8 + 2 * t;
    const bool vA = gA < geo.G;
    const bool vB = gA + 1 < geo.G;
    const int K8 = geo.K / 8;
#pragma unroll
    for (int rt = 0; rt < RT; ++rt) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = rb * geo.rows_per_block + rt * 16 + g + 8 * h;
            const bool vr = row < geo.N;
            const uint32_t* wr = p.w + static_cast<size_t>(row) * K8 + gA * 8;
            const uint4 z = make_uint4(0u, 0u, 0u, 0u);
            it.w[rt][h][0] = (vr && vA) ? ldg_stream(wr) : z;
            it.w[rt][h][1] = (vr && vA) ? ldg_stream(wr + 4) : z;
            it.w[rt][h][2] = (vr && vB) ? ldg_stream(wr + 8) : z;
            it.w[rt][h][3] = (vr && vB) ? ldg_stream(wr + 12) : z;
            const uint16_t* sr = reinterpret_cast<const uint16_t*>(p.s) + static_cast<size_t>(row) * geo.G + gA;
            const uint16_t* br = reinterpret_cast<const uint16_t*>(p.b) + static_cast<size_t>(row) * geo.G + gA;
            uint32_t s0 = (vr && vA) ? __ldg(sr) : 0u;
            uint32_t s1 = (vr && vB) ? __ldg(sr + 1) : 0u;
            uint32_t b0 = (vr && vA) ? __ldg(br) : 0u;
            uint32_t b1 = (vr && vB) ? __ldg(br + 1) : 0u;
            it.s[rt][h] = s0 | (s1 << 16);
            it.b[rt][h] = b0 | (b1 << 16);
        }
    }
}

__device__ __forceinline__ float block_sum(float v, float* tmp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) tmp[warp] = v;
    __syncthreads();
    float r = (lane < kWarps) ? tmp[lane] : 0.f;
    return warp_sum(r);
}

// bf16 GELU (tanh form) with the reference's per-op rounding; constants are bf16.
__device__ __forceinline__ float gelu_tanh_bf16ops(float x) {
    const float kC = 0.044677734375f;   // bf16(0.044715)
    const float kK = 0.796875f;         // bf16(sqrt(2/pi))
    float x2 = rbf(x * x);
    float x3 = rbf(x * x2);
    float in = rbf(kC * x3);
    in = rbf(in + x);
    in = rbf(kK * in);
    float th = rbf(tanhf(in));
    float hx = rbf(0.5f * x);
    float op = rbf(1.0f + th);
    return rbf(hx * op);
}

template <int RT>
__global__ void __launch_bounds__(kThreads, 1) qmv_kernel(const QmvParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;

    Geo geo;
    geo.K = p.K;
    geo.N = p.N;
    geo.G = p.K / 64;
    geo.nunits = (geo.G + 7) / 8;
    geo.rows_per_block = 16 * RT;
    geo.nrb = (p.N + geo.rows_per_block - 1) / geo.rows_per_block;

    // shared memory carve-up
    uint32_t* xp = reinterpret_cast<uint32_t*>(smem_raw);           // [K/2] permuted bf16 pairs
    uint32_t* zero_page = xp + geo.K / 2;                            // [32] zeros
    float* xsum = reinterpret_cast<float*>(zero_page + 32);          // [G] (+pad)
    float* red = xsum + ((geo.G + 3) & ~3);                          // [2][kWarps][16*RT]
    float* tmp = red + 2 * kWarps * 16 * RT;                         // [32]
    float* xf = tmp + 32;                                            // [K] staged activation (prologues)

    const int my_units = (warp < geo.nunits) ? (geo.nunits - warp + kWarps - 1) / kWarps : 0;
    const int my_rbs = (blockIdx.x < geo.nrb) ? (geo.nrb - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const int n_items = my_rbs * my_units;

    // the dependent kernel may launch at once: its PDL wait still waits for this grid
    pdl_launch_dependents();
    Item<RT> cur;
    if (n_items > 0) load_item<RT>(cur, p, geo, blockIdx.x, warp, g, t);

    // ---- wait for the producer of x, then stage the activation
    pdl_wait();
    if (threadIdx.x < 32) zero_page[threadIdx.x] = 0u;
    const int K = geo.K;
    if (p.prologue == QmvPrologue::kNone) {
        // build pairs directly from global x
        for (int gr = warp; gr < geo.G; gr += kWarps) {
            const uint16_t* xg = reinterpret_cast<const uint16_t*>(p.x) + gr * 64;
            const int i = lane >> 2, pp = lane & 3;
            uint16_t lo = xg[8 * i + pp], hi = xg[8 * i + pp + 4];
            xp[gr * 32 + lane] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
            float sv = warp_sum(bf2f(lo) + bf2f(hi));
            if (lane == 0) xsum[gr] = sv;
        }
    } else {
        float ss = 0.f;
        for (int k = threadIdx.x; k < K; k += kThreads) {
            float v = bf2f(p.x[k]);
            xf[k] = v;
            ss += v * v;
        }
        float tot = block_sum(ss, tmp);
        float inv = 1.0f / sqrtf(tot / static_cast<float>(K) + p.eps);
        if (p.prologue == QmvPrologue::kResidNorm) {
            float ss2 = 0.f;
            const float sc = p.scalar ? bf2f(p.scalar[0]) : 1.0f;
            for (int k = threadIdx.x; k < K; k += kThreads) {
                float nv = rbf(rbf(xf[k] * inv) * bf2f(p.post_w[k]));
                float hv = rbf(bf2f(p.resid[k]) + nv);
                if (p.scalar) hv = rbf(hv * sc);
                xf[k] = hv;
                ss2 += hv * hv;
                if (blockIdx.x == 0 && p.h_out) p.h_out[k] = f2bf(hv);
            }
            tot = block_sum(ss2, tmp);
            inv = 1.0f / sqrtf(tot / static_cast<float>(K) + p.eps);
        }
        for (int k = threadIdx.x; k < K; k += kThreads) {
            xf[k] = rbf(rbf(xf[k] * inv) * bf2f(p.norm_w[k]));
        }
        __syncthreads();
        for (int gr = warp; gr < geo.G; gr += kWarps) {
            const float* xg = xf + gr * 64;
            const int i = lane >> 2, pp = lane & 3;
            float lo = xg[8 * i + pp], hi = xg[8 * i + pp + 4];
            xp[gr * 32 + lane] = pack_bf2(f2bf(lo), f2bf(hi));
            float sv = warp_sum(lo + hi);
            if (lane == 0) xsum[gr] = sv;
        }
    }
    __syncthreads();

    int buf = 0;
    int it = 0;
    for (int ri = 0; ri < my_rbs; ++ri) {
        const int rb = blockIdx.x + ri * gridDim.x;
        float acc[RT][2];
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) acc[rt][0] = acc[rt][1] = 0.f;

        for (int ui = 0; ui < my_units; ++ui, ++it) {
            const int unit = warp + ui * kWarps;
            Item<RT> nxt;
            if (it + 1 < n_items) {
                const int ni = it + 1;
                const int nrb = blockIdx.x + (ni / my_units) * gridDim.x;
                const int nun = warp + (ni % my_units) * kWarps;
                load_item<RT>(nxt, p, geo, nrb, nun, g, t);
            }
            const int gA = unit * 8 + 2 * t;
            // B sources: lane g == 2t carries group gA in b0, lane g == 2t+1 carries gB in b1.
            const uint32_t* src0 = (g == 2 * t && gA < geo.G) ? xp + gA * 32 : zero_page;
            const uint32_t* src1 = (g == 2 * t + 1 && gA + 1 < geo.G) ? xp + (gA + 1) * 32 : zero_page;
            float d[RT][4];
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) d[rt][0] = d[rt][1] = d[rt][2] = d[rt][3] = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 b0v = *reinterpret_cast<const uint4*>(src0 + 4 * i);
                const uint4 b1v = *reinterpret_cast<const uint4*>(src1 + 4 * i);
                const uint32_t b0s[4] = {b0v.x, b0v.y, b0v.z, b0v.w};
                const uint32_t b1s[4] = {b1v.x, b1v.y, b1v.z, b1v.w};
#pragma unroll
                for (int rt = 0; rt < RT; ++rt) {
                    // word i of group A / B for rows g (h=0) and g+8 (h=1)
                    const uint4* wa0 = &cur.w[rt][0][i >> 2];
                    const uint4* wa1 = &cur.w[rt][1][i >> 2];
                    const uint4* wb0 = &cur.w[rt][0][2 + (i >> 2)];
                    const uint4* wb1 = &cur.w[rt][1][2 + (i >> 2)];
                    const int c = i & 3;
                    const uint32_t xa0 = c == 0 ? wa0->x : c == 1 ? wa0->y : c == 2 ? wa0->z : wa0->w;
                    const uint32_t xa1 = c == 0 ? wa1->x : c == 1 ? wa1->y : c == 2 ? wa1->z : wa1->w;
                    const uint32_t xb0 = c == 0 ? wb0->x : c == 1 ? wb0->y : c == 2 ? wb0->z : wb0->w;
                    const uint32_t xb1 = c == 0 ? wb1->x : c == 1 ? wb1->y : c == 2 ? wb1->z : wb1->w;
#pragma unroll
                    for (int pp = 0; pp < 4; ++pp) {
                        const uint32_t a0 = lop3_and_or(xa0 >> (4 * pp), 0x000F000Fu, 0x43004300u);
                        const uint32_t a1 = lop3_and_or(xa1 >> (4 * pp), 0x000F000Fu, 0x43004300u);
                        const uint32_t a2 = lop3_and_or(xb0 >> (4 * pp), 0x000F000Fu, 0x43004300u);
                        const uint32_t a3 = lop3_and_or(xb1 >> (4 * pp), 0x000F000Fu, 0x43004300u);
                        mma_bf16_16816(d[rt], a0, a1, a2, a3, b0s[pp], b1s[pp]);
                    }
                }
            }
            // fold the group dots with their scales and biases
            const float xsA = (gA < geo.G) ? xsum[gA] : 0.f;
            const float xsB = (gA + 1 < geo.G) ? xsum[gA + 1] : 0.f;
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float sA = __uint_as_float(cur.s[rt][h] << 16);
                    const float sB = __uint_as_float(cur.s[rt][h] & 0xFFFF0000u);
                    const float bA = __uint_as_float(cur.b[rt][h] << 16);
                    const float bB = __uint_as_float(cur.b[rt][h] & 0xFFFF0000u);
                    float a = acc[rt][h];
                    a = fmaf(sA, d[rt][2 * h + 0], a);
                    a = fmaf(sB, d[rt][2 * h + 1], a);
                    a = fmaf(fmaf(-128.f, sA, bA), xsA, a);
                    a = fmaf(fmaf(-128.f, sB, bB), xsB, a);
                    acc[rt][h] = a;
                }
            }
            cur = nxt;
        }
        // reduce over the four t lanes, then across warps
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float v = acc[rt][h];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if (t == 0) red[(buf * kWarps + warp) * 16 * RT + rt * 16 + g + 8 * h] = v;
            }
        }
        __syncthreads();
        if (p.epilogue == QmvEpilogue::kStore) {
            if (threadIdx.x < 16 * RT) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) v += red[(buf * kWarps + w) * 16 * RT + threadIdx.x];
                const int row = rb * geo.rows_per_block + threadIdx.x;
                if (row < geo.N) p.y[row] = f2bf(v);
            }
        } else {
            // rows [0,16) of the block are gate rows, [16,32) the matching up rows
            if (RT == 2 && threadIdx.x < 16) {
                float gv = 0.f, uv = 0.f;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) {
                    gv += red[(buf * kWarps + w) * 16 * RT + threadIdx.x];
                    uv += red[(buf * kWarps + w) * 16 * RT + 16 + threadIdx.x];
                }
                const int row = rb * 16 + threadIdx.x;
                if (row < geo.N / 2) p.y[row] = f2bf(gelu_tanh_bf16ops(rbf(gv)) * rbf(uv));
            }
        }
        buf ^= 1;
    }
}

size_t qmv_smem_bytes(int K, int RT, bool prologue) {
    const int G = K / 64;
    size_t b = static_cast<size_t>(K / 2) * 4 + 32 * 4 + static_cast<size_t>((G + 3) & ~3) * 4 +
               static_cast<size_t>(2 * kWarps * 16 * RT) * 4 + 32 * 4;
    if (prologue) b += static_cast<size_t>(K) * 4;
    return b;
}

template <int RT>
void launch_rt(const QmvParams& p, cudaStream_t stream, bool pdl) {
    const bool pro = p.prologue != QmvPrologue::kNone;
    const size_t smem = qmv_smem_bytes(p.K, RT, pro);
    static bool attr_set[2] = {false, false};
    if (smem > 48 * 1024 && !attr_set[RT - 1]) {
        HYB_CUDA(cudaFuncSetAttribute(qmv_kernel<RT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      227 * 1024));
        attr_set[RT - 1] = true;
    }
    const int nrb = (p.N + 16 * RT - 1) / (16 * RT);
    const int grid = std::max(1, std::min(nrb, num_sms() * (RT == 1 ? 2 : 1)));
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
    HYB_CUDA(cudaLaunchKernelEx(&cfg, qmv_kernel<RT>, p));
}

}  // namespace

void launch_qmv(const QmvParams& p, cudaStream_t stream, bool pdl) {
    if (p.packed) {  // packed resident layout: the TMA-streamed kernel
        launch_qmv_packed(p, stream, pdl);
        return;
    }
    if (p.K <= 0 || p.K % 64 != 0 || p.N <= 0) throw ArgError("qmv: K must be a positive multiple of 64");
    if (p.epilogue == QmvEpilogue::kGeglu) {
        if (p.N % 32 != 0) throw ArgError("qmv geglu: interleaved rows must be a multiple of 32");
        launch_rt<2>(p, stream, pdl);
        return;
    }
    // Two row tiles per warp when there are enough rows to keep every SM busy.
    const int nrb2 = (p.N + 31) / 32;
    if (nrb2 >= 2 * num_sms()) {
        launch_rt<2>(p, stream, pdl);
    } else {
        launch_rt<1>(p, stream, pdl);
    }
}

}  // namespace hyb
